"""The reference-facing hot-expert method and hot cache on the GPU.

KTGGUFHotExpertsMethod is built as the KT wrapper builds it (hot/kt_gguf_hot.py:163-304):
create_weights, process_weights_after_loading from a GGUF reader (a fake in `_readers`
serving synthetic experts), then apply() on a dispatch output. Prefill-sized chunks run
the tcgen05 layer (checked against the fp32 dequant-then-matmul oracle, rel-L2 <= 5e-3);
decode windows run the q8_1 GEMV path (checked against the restated reference layer).
HotCache.route is checked against table gathers and an exact count histogram."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from kt_gguf_b200 import kt_gguf_hot as H
from kt_gguf_b200 import kt_hot_cache as C
from kt_gguf_b200 import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL_FP32_ORACLE = 5e-3  # north-star bound, bf16 activations
TOL_REF_LAYER = 2e-3    # GEMV path vs the restated reference layer (same q8_1 / bf16 arithmetic)


class FakeGGUF:
    """Serves one synthetic layer's experts the way _GGUFExperts serves a GGUF file."""

    def __init__(self, L: synth.MoELayer):
        self.L = L
        self.E, self.inter, self.K = L.w13.shape[0], L.inter, L.hidden

    def types(self, layer_idx):
        return (self.L.type13, self.L.type13, self.L.type2)

    def slice(self, layer_idx, proj, N, rank, experts):
        e = experts.numpy()
        if proj == "gate":
            v = self.L.w13[e, :N]
        elif proj == "up":
            v = self.L.w13[e, N:]
        else:
            v = self.L.w2[e]
        return torch.from_numpy(np.ascontiguousarray(v))


def build_method(L: synth.MoELayer, key: str):
    H._readers[key] = FakeGGUF(L)
    kt = SimpleNamespace(num_gpu_experts=L.w13.shape[0], weight_path=key, layer_idx=0)
    layer = torch.nn.Module()
    layer.moe_tp_rank, layer.moe_tp_size = 0, 1
    m = H.KTGGUFHotExpertsMethod(kt, layer)
    m.create_weights(layer, L.w13.shape[0], L.hidden, L.inter, torch.bfloat16)
    m.process_weights_after_loading(layer)
    m.create_moe_runner(layer, None)
    return m, layer


def apply(m, layer, L, dev):
    d = SimpleNamespace(hidden_states=L.x.to(dev), topk_output=(L.topk_weights.to(dev), L.topk_ids.to(dev), None))
    out = m.apply(layer, d).hidden_states
    torch.cuda.synchronize()
    return out


def test_hot_method_loads_slots_from_reader(cuda_device):
    L = synth.make_layer(11, 8, 2048, 512, 32, 8, 12, 14, n_hot=8)
    m, layer = build_method(L, "fake://load")
    assert torch.equal(layer.w13_qweight.cpu(), torch.from_numpy(L.w13))
    assert torch.equal(layer.w2_qweight.cpu(), torch.from_numpy(L.w2))
    assert (m.type13, m.type2) == (12, 14)


@pytest.mark.parametrize("type13,type2", [(12, 14), (8, 8), (21, 21)])
def test_hot_method_prefill_chunk(cuda_device, type13, type2):
    L = synth.make_layer(5, 384, 2048, 512, 48, 8, type13, type2, n_hot=24, zipf=1.1)
    m, layer = build_method(L, f"fake://prefill{type13}")
    assert m._use_prefill(L.x, 384)
    out = apply(m, layer, L, cuda_device)
    want = O.moe_fp32(L.x.view(torch.int16).numpy().view(np.uint16), L.topk_ids.numpy(), L.topk_weights.numpy(),
                      type13, L.w13, type2, L.w2, L.inter)
    err = O.rel_l2(out.float().cpu().numpy(), want)
    assert err <= TOL_FP32_ORACLE, err


@pytest.mark.parametrize("tokens", [1, 4, 16])
def test_hot_method_decode_window(cuda_device, tokens):
    L = synth.make_layer(7, tokens, 2048, 512, 32, 8, 12, 14, n_hot=16)
    m, layer = build_method(L, f"fake://decode{tokens}")
    assert not m._use_prefill(L.x, tokens)
    out = apply(m, layer, L, cuda_device)
    x16 = L.x.view(torch.int16).numpy().view(np.uint16)
    ref = O.bf16_to_f32(O.moe_ref_bf16(x16, L.topk_ids.numpy(), L.topk_weights.numpy(), 12, L.w13, 14, L.w2, L.inter))
    err = O.rel_l2(out.float().cpu().numpy(), ref)
    assert err <= TOL_REF_LAYER, err


@pytest.mark.parametrize("tokens", [4, 384])
def test_hot_method_q2_0_native_down(cuda_device, monkeypatch, tokens):
    # hot/kt_gguf_hot.py:21-25, 180-190: a Q2_0 down stays 2-bit and the layer runs the GEMV at
    # every length (a prefill-sized chunk included)
    monkeypatch.setenv("KT_GGUF_Q2_NATIVE", "1")
    L = synth.make_layer(9, tokens, 2048, 512, 32, 8, 12, 42, n_hot=16, zipf=1.1)
    m, layer = build_method(L, f"fake://q2native{tokens}")
    assert m.type2 == 42 and not m._use_prefill(L.x, tokens)
    assert torch.equal(layer.w2_qweight.cpu(), torch.from_numpy(L.w2))
    out = apply(m, layer, L, cuda_device)
    x16 = L.x.view(torch.int16).numpy().view(np.uint16)
    ref = O.bf16_to_f32(O.moe_ref_bf16(x16, L.topk_ids.numpy(), L.topk_weights.numpy(), 12, L.w13, 42, L.w2, L.inter))
    err = O.rel_l2(out.float().cpu().numpy(), ref)
    assert err <= TOL_REF_LAYER, err


def test_hot_method_q2_0_repacked_down_prefill(cuda_device, monkeypatch):
    # KT_GGUF_Q2_NATIVE=0: the exact Q8_0 repack, which the tcgen05 prefill layer takes
    monkeypatch.setenv("KT_GGUF_Q2_NATIVE", "0")
    L = synth.make_layer(9, 384, 2048, 512, 32, 8, 12, 42, n_hot=16, zipf=1.1)
    m, layer = build_method(L, "fake://q2repack")
    assert m.type2 == 8 and m._use_prefill(L.x, 384)
    out = apply(m, layer, L, cuda_device)
    want = O.moe_fp32(L.x.view(torch.int16).numpy().view(np.uint16), L.topk_ids.numpy(), L.topk_weights.numpy(),
                      12, L.w13, 42, L.w2, L.inter)  # the Q2_0 values themselves: the repack is exact
    err = O.rel_l2(out.float().cpu().numpy(), want)
    assert err <= TOL_FP32_ORACLE, err


def test_hot_cache_route_on_gpu(cuda_device):
    E, NS = 64, 16
    c = C.HotCache(1, E, NS, cuda_device, 0)
    c.layers[0] = (None, None)
    perm = np.random.default_rng(2).permutation(E)[:NS]
    for s, e in enumerate(perm.tolist()):
        c._set(0, s, e)
    c.push_tables()
    assert c.check_tables() == ""
    g = torch.Generator().manual_seed(4)
    for T in (1, 4, 700):  # decode window and a long extend (one kernel at every size)
        ids = torch.stack([torch.randperm(E, generator=g)[:8] for _ in range(T)]).to(torch.int32)
        before = c.counts.clone()
        slot, cpu = c.route(0, ids.to(cuda_device))
        torch.cuda.synchronize()
        assert torch.equal(slot.cpu(), c.log2slot_cpu[0][ids.long()])
        assert torch.equal(cpu.cpu(), c.log2cpu_cpu[0][ids.long()])
        hist = torch.bincount(ids.reshape(-1).long(), minlength=E).float()
        assert torch.equal((c.counts - before)[0].cpu(), hist)


class _DecodeMode:
    @staticmethod
    def is_decode():
        return True

    @staticmethod
    def is_target_verify():
        return False


def test_dynamic_swap_then_layer_matches_oracle(cuda_device, tmp_path, monkeypatch):
    # The whole decode-adaptive path on a real GGUF file: the hot method loads experts 0 and 1
    # into its two slots; decode routes make expert 4 hot; before_forward swaps it in (the counts
    # of a policy round come back one round late); then the layer, routed through the cache's
    # tables, must equal the oracle on the logical experts that are now resident.
    from gguf_fixture import E, INTER, K, write_gguf

    monkeypatch.setattr(C, "INTERVAL", 1)
    monkeypatch.setattr(C, "KV_LEND", False)
    path = tmp_path / "experts.gguf"
    data = write_gguf(path, seed=7)
    H._readers.pop(str(path), None)
    kt = SimpleNamespace(num_gpu_experts=2, weight_path=str(path), layer_idx=0, num_layers=1)
    layer = torch.nn.Module()
    layer.moe_tp_rank, layer.moe_tp_size = 0, 1
    m = H.KTGGUFHotExpertsMethod(kt, layer)
    m.create_weights(layer, 2, K, INTER, torch.bfloat16)
    m.process_weights_after_loading(layer)
    dev = cuda_device
    c = C.HotCache(1, E, 2, dev, 0)
    c.layers[0] = (m, layer)
    c.seed(None)
    assert c.slot2log[0] == [0, 1]
    g = torch.Generator().manual_seed(5)
    hot = torch.tensor([[4, 0], [4, 2], [4, 5], [3, 4]], dtype=torch.int32).to(dev)
    batch = SimpleNamespace(forward_mode=_DecodeMode())
    for _ in range(3):
        c.route(0, hot)  # expert 4: 4 routes a step; expert 0: 1; expert 1: none
        c.before_forward(batch)
    torch.cuda.synchronize()
    assert c.swaps >= 1 and 4 in c.slot2log[0] and c.check_tables() == ""
    s4 = c.slot2log[0].index(4)
    assert s4 == 1  # the colder slot (expert 1) gave way
    w13_all = np.concatenate([data[(0, "gate")], data[(0, "up")]], axis=1)
    w2_all = data[(0, "down")]
    assert torch.equal(layer.w13_qweight[s4].cpu(), torch.from_numpy(w13_all[4]))
    assert torch.equal(layer.w2_qweight[s4].cpu(), torch.from_numpy(w2_all[4]))
    for T in (4, 256):  # a decode window (GEMV path) and a prefill chunk (tcgen05 path)
        logical = torch.stack([torch.randperm(E, generator=g)[:2] for _ in range(T)]).to(torch.int32)
        slot_ids, cpu_ids = c.route(0, logical.to(dev))
        x = torch.randn((T, K), generator=g).to(torch.bfloat16)
        w = torch.rand((T, 2), generator=g)
        d = SimpleNamespace(hidden_states=x.to(dev), topk_output=(w.to(dev), slot_ids, None))
        out = m.apply(layer, d).hidden_states.float().cpu().numpy()
        res = slot_ids.cpu() >= 0
        assert torch.equal(res, cpu_ids.cpu() < 0)  # each route on exactly one side
        masked = torch.where(res, logical, torch.full_like(logical, -1)).numpy()
        xb = x.view(torch.int16).numpy().view(np.uint16)
        if T == 4:
            want = O.bf16_to_f32(O.moe_ref_bf16(xb, masked, w.numpy(), 12, w13_all, 14, w2_all, INTER))
            assert O.rel_l2(out, want) <= TOL_REF_LAYER
        else:
            want = O.moe_fp32(xb, masked, w.numpy(), 12, w13_all, 14, w2_all, INTER)
            assert O.rel_l2(out, want) <= TOL_FP32_ORACLE
