"""The streamed prefill of non-resident experts (kt_stream_prefill_gguf.KTStreamPrefillGGUF)
and its C-ABI group call (kt_moe_prefill_ex) on the GPU.

Follows the reference's streamer (the flash-next-gguf SGLang tree, kt_stream_prefill_gguf.py:
KTStreamPrefillGGUF.run / _stage / _group_body): experts from num_gpu_experts on, in groups,
raw GGUF bytes staged from pinned banks, one fused MoE per group, summed over the groups.
Checked against the fp32 dequant-then-matmul oracle restricted to the streamed experts
(rel-L2 <= 5e-3, the north-star bound for bf16 activations)."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from kt_gguf_b200 import _native as N
from kt_gguf_b200 import kt_gguf_moe_multi as M
from kt_gguf_b200 import kt_stream_prefill_gguf as SP
from kt_gguf_b200 import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL_FP32_ORACLE = 5e-3


class Reader:
    """The hot method's GGUF reader over a synthetic layer of E experts (physical order)."""

    def __init__(self, L: synth.MoELayer):
        self.L = L
        self.E = L.w13.shape[0]

    def types(self, layer_idx):
        return (self.L.type13, self.L.type13, self.L.type2)

    def slice(self, layer_idx, proj, N_, rank, experts):
        e = experts.numpy()
        v = {"gate": self.L.w13[e, :N_], "up": self.L.w13[e, N_:], "down": self.L.w2[e]}[proj]
        return torch.from_numpy(np.ascontiguousarray(v))


def method_for(L, n_gpu):
    return SimpleNamespace(reader=Reader(L), rank=0, world=1, N=L.inter, K=L.hidden, num_gpu_experts=n_gpu,
                           kt_config=SimpleNamespace(layer_idx=0), streams_hot_experts=False)


def dispatch(L, dev):
    return SimpleNamespace(hidden_states=L.x.to(dev), topk_output=SimpleNamespace(topk_weights=L.topk_weights.to(dev)))


def oracle_streamed(L, n_gpu):
    ids = L.topk_ids.numpy().copy()
    ids[ids < n_gpu] = -1  # the resident experts are the hot method's
    x16 = L.x.view(torch.int16).numpy().view(np.uint16)
    return O.moe_fp32(x16, ids, L.topk_weights.numpy(), L.type13, L.w13, L.type2, L.w2, L.inter)


@pytest.fixture(scope="module")
def layer40():
    # 40 experts, all with weights (n_hot None: ids are the physical ids), 8 of them resident
    return synth.make_layer(21, 640, 2048, 512, 40, 8, 12, 14)


@pytest.mark.parametrize("G", [8, 5, 32])
def test_streamed_experts_match_oracle(cuda_device, layer40, G):
    L = layer40
    sp = SP.KTStreamPrefillGGUF(method_for(L, 8), group_size=G)
    assert sp.groups(8) == [(b, min(G, 40 - b)) for b in range(8, 40, G)]
    out = sp.run(method_for(L, 8), None, dispatch(L, cuda_device), L.topk_ids.to(cuda_device))
    torch.cuda.synchronize()
    want = oracle_streamed(L, 8)
    err = O.rel_l2(out.float().cpu().numpy(), want)
    assert err <= TOL_FP32_ORACLE, err
    pb = sp._part_bytes[0]
    assert sp.bytes_staged == 32 * (pb[0] + pb[1])  # every streamed expert crossed once


def test_group_size_changes_only_the_fp32_order(cuda_device, layer40):
    L = layer40
    outs = []
    for G in (32, 8, 3):
        sp = SP.KTStreamPrefillGGUF(method_for(L, 8), group_size=G)
        outs.append(sp.run(method_for(L, 8), None, dispatch(L, cuda_device), L.topk_ids.to(cuda_device)).float())
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert O.rel_l2(o.cpu().numpy(), outs[0].cpu().numpy()) < 2e-3


def test_window_equals_remapped_slots(cuda_device, layer40):
    # kt_moe_prefill_ex on slots [8, 16) with id_base 8 == kt_moe_prefill with the ids remapped
    L = layer40
    x, w = L.x.to(cuda_device), L.topk_weights.to(cuda_device)
    ids = L.topk_ids.to(cuda_device)
    w13 = torch.from_numpy(L.w13[8:16]).to(cuda_device)
    w2 = torch.from_numpy(L.w2[8:16]).to(cuda_device)
    a = M.moe_prefill_ex(x, w13, w2, ids, w, 12, 14, L.inter, id_base=8)
    remap = torch.where((ids >= 8) & (ids < 16), ids - 8, torch.full_like(ids, -1))
    b = M.moe_prefill(x, w13, w2, remap, w, 12, 14, L.inter)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_accumulator_flags(cuda_device, layer40):
    L = layer40
    dev = cuda_device
    x, w, ids = L.x.to(dev), L.topk_weights.to(dev), L.topk_ids.to(dev)
    w13 = torch.from_numpy(L.w13).to(dev)
    w2 = torch.from_numpy(L.w2).to(dev)
    T, K = x.shape
    whole = M.moe_prefill_ex(x, w13, w2, ids, w, 12, 14, L.inter)
    acc = torch.full((T, K), float("nan"), dtype=torch.float32, device=dev)
    M.moe_prefill_ex(x, w13[:16], w2[:16], ids, w, 12, 14, L.inter, id_base=0, acc=acc, acc_flags=N.KT_ACC_STORE)
    assert not torch.isnan(acc).any()  # STORE alone writes every token
    snap = acc.clone()
    # a group none of whose experts is routed to leaves acc bit for bit (tokens skipped)
    M.moe_prefill_ex(x, w13[39:40], w2[39:40], torch.zeros_like(ids) - 1, w, 12, 14, L.inter, id_base=39, acc=acc,
                     acc_flags=N.KT_ACC_LOAD | N.KT_ACC_STORE)
    assert torch.equal(acc, snap)
    M.moe_prefill_ex(x, w13[16:32], w2[16:32], ids, w, 12, 14, L.inter, id_base=16, acc=acc,
                     acc_flags=N.KT_ACC_LOAD | N.KT_ACC_STORE)
    out = M.moe_prefill_ex(x, w13[32:], w2[32:], ids, w, 12, 14, L.inter, id_base=32, acc=acc,
                           acc_flags=N.KT_ACC_LOAD)
    torch.cuda.synchronize()
    # the same sum in another fp32 order, rounded once: one bf16 ulp apart at most (2^-7 of the
    # value), plus 1e-5 of the row's largest magnitude where the sum cancels
    a, b = out.float(), whole.float()
    slack = 1e-5 * b.abs().amax(dim=1, keepdim=True)
    assert bool(((a - b).abs() <= b.abs() * 2.0 ** -7 + slack).all())
    assert float((out != whole).float().mean()) < 0.05
    x16 = L.x.view(torch.int16).numpy().view(np.uint16)
    want = O.moe_fp32(x16, L.topk_ids.numpy(), L.topk_weights.numpy(), 12, L.w13, 14, L.w2, L.inter)
    assert O.rel_l2(out.float().cpu().numpy(), want) <= TOL_FP32_ORACLE


def test_hot_plus_streamed_is_the_whole_layer(cuda_device, layer40):
    # the resident experts through the prefill layer on their slots, the rest streamed: their
    # sum is the layer over every expert
    L = layer40
    dev = cuda_device
    ids = L.topk_ids.to(dev)
    slot_ids = torch.where(ids < 8, ids, torch.full_like(ids, -1))
    hot = M.moe_prefill(L.x.to(dev), torch.from_numpy(L.w13[:8]).to(dev), torch.from_numpy(L.w2[:8]).to(dev), slot_ids,
                        L.topk_weights.to(dev), 12, 14, L.inter)
    sp = SP.KTStreamPrefillGGUF(method_for(L, 8), group_size=8)
    streamed = sp.run(method_for(L, 8), None, dispatch(L, dev), ids)
    total = hot.float() + streamed.float()
    torch.cuda.synchronize()
    x16 = L.x.view(torch.int16).numpy().view(np.uint16)
    want = O.moe_fp32(x16, L.topk_ids.numpy(), L.topk_weights.numpy(), 12, L.w13, 14, L.w2, L.inter)
    assert O.rel_l2(total.cpu().numpy(), want) <= TOL_FP32_ORACLE


def test_nothing_to_stream(cuda_device, layer40):
    L = layer40
    m = method_for(L, 40)  # every expert resident
    sp = SP.KTStreamPrefillGGUF(m, group_size=8)
    out = sp.run(m, None, dispatch(L, cuda_device), L.topk_ids.to(cuda_device))
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0 and sp.bytes_staged == 0


def test_stream_self_check_reports_parity(cuda_device, layer40, monkeypatch):
    # KT_GPU_STREAM_SELFTEST=2: the first streamed layer is recomputed by fp32 dequant + matmul
    # (the reference's _reference_check) and the result kept; later calls do not check again
    monkeypatch.setattr(SP, "SELFTEST", "2")
    L = layer40
    sp = SP.KTStreamPrefillGGUF(method_for(L, 8), group_size=16)
    out = sp.run(method_for(L, 8), None, dispatch(L, cuda_device), L.topk_ids.to(cuda_device))
    chk = sp.last_check
    assert chk is not None and chk["experts_used"] == 32 and chk["tokens"] == L.x.shape[0]
    assert chk["rel_l2"] <= TOL_FP32_ORACLE and chk["cosine"] > 0.9999
    want = oracle_streamed(L, 8)
    assert O.rel_l2(out.float().cpu().numpy(), want) <= TOL_FP32_ORACLE
    sp.run(method_for(L, 8), None, dispatch(L, cuda_device), L.topk_ids.to(cuda_device))
    assert sp.last_check is chk
