"""Host logic of the decode-adaptive hot cache (kt_hot_cache.HotCache) and the hot method's
helpers, on CPU tensors: seeding, residency invariants, the swap policy, slot filling from
the banks, KV-lent slots, and the exact Q2_0 -> Q8_0 repack. Follows the behaviour of
hot/kt_hot_cache.py:184-460 and hot/kt_gguf_hot.py (q2_0_to_q8_0)."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from kt_gguf_b200 import kt_gguf_hot as H
from kt_gguf_b200 import kt_hot_cache as C
from oracle import oracle as O

L, E, NS, N_INTER, ROWB13, ROWB2 = 2, 16, 4, 8, 36, 20


class FakeReader:
    """Expert e of layer l: every byte = (l * 64 + e * 3 + proj) & 255."""

    def __init__(self):
        self.E = E

    def slice(self, li, proj, N, rank, experts):
        p = ("gate", "up", "down").index(proj)
        cols = N if proj != "down" else 2 * N
        rb = ROWB13 if proj != "down" else ROWB2
        v = torch.empty((len(experts), cols, rb), dtype=torch.uint8)
        for i, e in enumerate(experts.tolist()):
            v[i] = (li * 64 + e * 3 + p) & 255
        return v


def make_cache(kv_lend=False, monkeypatch=None):
    if monkeypatch is not None:
        monkeypatch.setattr(C, "KV_LEND", kv_lend)
        monkeypatch.setattr(C, "KV_LEND_MAX", 2)
    c = C.HotCache(L, E, NS, torch.device("cpu"), 0)
    rd = FakeReader()
    for li in range(L):
        method = SimpleNamespace(reader=rd, N=N_INTER, rank=0, types=(12, 12, 14), type2=14)
        layer = SimpleNamespace(w13_qweight=torch.zeros((NS, 2 * N_INTER, ROWB13), dtype=torch.uint8),
                                w2_qweight=torch.zeros((NS, 2 * N_INTER, ROWB2), dtype=torch.uint8))
        c.layers[li] = (method, layer)
    return c


def slot_bytes(c, li, s):
    _m, layer = c.layers[li]
    if s >= c.N:
        v13, v2 = c.lent_views[(li, s)]
    else:
        v13, v2 = layer.w13_qweight[s], layer.w2_qweight[s]
    return int(v13[0, 0]), int(v13[N_INTER, 0]), int(v2[0, 0])


def expect_bytes(li, e):
    return tuple((li * 64 + e * 3 + p) & 255 for p in range(3))


def test_seed_logical_order_and_invariants(monkeypatch):
    c = make_cache(monkeypatch=monkeypatch)
    c.seed(None)
    assert c.ready and c.check_tables() == ""
    for li in range(L):
        assert c.log2slot_cpu[li, :NS].tolist() == list(range(NS))
        assert (c.log2slot_cpu[li, NS:] == -1).all()
        assert (c.log2cpu_cpu[li, :NS] == -1).all()
        assert c.log2cpu_cpu[li, NS:].tolist() == list(range(NS, E))


def test_check_tables_finds_violations(monkeypatch):
    c = make_cache(monkeypatch=monkeypatch)
    c.seed(None)
    c.log2cpu_cpu[1, 7] = -1  # neither on a slot nor on the CPU
    c.push_tables()
    assert "neither" in c.check_tables()
    c.log2cpu_cpu[1, 7] = 7
    c.push_tables()
    c.log2cpu[0, 9] = 3  # device table differs from the host's
    assert "differ" in c.check_tables()


def test_plan_swaps_policy(monkeypatch):
    monkeypatch.setattr(C, "MAX_SWAPS", 3)
    monkeypatch.setattr(C, "MARGIN", 1.5)
    c = make_cache(monkeypatch=monkeypatch)
    c.seed(None)
    counts = torch.zeros((L, E))
    counts[0, :NS] = torch.tensor([5.0, 1.0, 9.0, 2.0])  # residents of layer 0
    counts[0, 10], counts[0, 11], counts[0, 12] = 20.0, 2.9, 1.0
    counts[1, :NS] = 4.0
    counts[1, 15] = 6.0  # 6 <= 1.5 * 4: no swap in layer 1
    plan = C.HotCache.plan_swaps(c, counts)
    # coldest resident slot 1 (1.0) <- 10 (20.0); next slot 3 (2.0) <- 11 (2.9 < 3.0 stops the chain)
    assert plan == [(0, 1, 10)]
    for li, s, e in plan:
        c._set(li, s, e)
        c.fill(li, s, e)
    c.push_tables()
    assert c.check_tables() == ""
    assert int(c.log2slot_cpu[0, 10]) == 1 and int(c.log2cpu_cpu[0, 1]) == 1
    assert slot_bytes(c, 0, 1) == expect_bytes(0, 10)


def test_plan_swaps_chain_and_empty_slots(monkeypatch):
    monkeypatch.setattr(C, "MAX_SWAPS", 8)
    c = make_cache(monkeypatch=monkeypatch)
    c._set(0, 0, 0)  # layer 0: slots 1..3 EMPTY; layer 1 all EMPTY
    counts = torch.zeros((L, E))
    counts[0, 5], counts[0, 6] = 3.0, 0.5
    plan = C.HotCache.plan_swaps(c, counts)
    # EMPTY slots score -1 and take any candidate seen at all (count > 0); zero counts never swap in
    assert sorted(plan) == [(0, 1, 5), (0, 2, 6)]


def test_fill_empty_and_lent_slots(monkeypatch):
    c = make_cache(kv_lend=True, monkeypatch=monkeypatch)
    c.seed(None)
    assert c.S == NS + 2 and c.slot2log[0][NS:] == [C.ABSENT, C.ABSENT]
    v13 = torch.zeros((2 * N_INTER, ROWB13), dtype=torch.uint8)
    v2 = torch.zeros((2 * N_INTER, ROWB2), dtype=torch.uint8)
    c.lend_slot(0, NS, v13, v2)
    with pytest.raises(RuntimeError):
        c.lend_slot(0, NS, v13, v2)
    counts = torch.zeros((L, E))
    counts[0, 13] = 7.0
    assert c.fill_empty(counts) == 1
    c.push_tables()
    assert c.check_tables() == ""
    assert slot_bytes(c, 0, NS) == expect_bytes(0, 13)
    # full tables: 13 on the lent slot; base tables: 13 stays on the CPU
    assert int(c.log2slot_cpu[0, 13]) == NS and int(c.log2cpu_cpu[0, 13]) == -1
    assert int(c.log2slot_base_cpu[0, 13]) == -1 and int(c.log2cpu_base_cpu[0, 13]) == 13
    assert c.take_back_slot(0, NS) == 13
    c.push_tables()
    assert c.check_tables() == "" and int(c.log2cpu_cpu[0, 13]) == 13
    with pytest.raises(RuntimeError):
        c.take_back_slot(0, NS)


def test_fill_empty_seed_rank_breaks_ties(monkeypatch):
    c = make_cache(monkeypatch=monkeypatch)
    counts = torch.zeros((L, E))
    seed_rank = torch.arange(E).flip(0).repeat(L, 1)  # the map prefers the highest ids
    assert c.fill_empty(counts, seed_rank) == L * NS
    assert sorted(c.slot2log[0]) == list(range(E - NS, E))


def test_q2_0_repack_is_exact():
    rng = np.random.default_rng(3)
    n = 64
    blocks = rng.integers(0, 256, size=(n, 18), dtype=np.uint8)
    blocks[:, :2] = np.frombuffer(rng.uniform(-1, 1, n).astype(np.float16).tobytes(), dtype=np.uint8).reshape(n, 2)
    d = blocks[:, :2].copy().view(np.float16).astype(np.float32).reshape(n)
    codes = ((blocks[:, 2:, None] >> np.array([0, 2, 4, 6], dtype=np.uint8)) & 3).reshape(n, 64).astype(np.float32)
    want = d[:, None] * (codes - 1)
    q8 = H.q2_0_to_q8_0(torch.from_numpy(blocks.reshape(1, -1))).numpy()
    assert q8.shape == (1, n * 68)
    got = O.dequant(8, q8, n * 64).reshape(n, 64)
    assert np.array_equal(got, want)


def test_q2_0_oracle_dequant_equals_the_q8_0_repack():
    # the Q2_0 decoder of the oracle against an independent route: the exact Q8_0 repack,
    # decoded by the Q8_0 path that gguf-py's golden vectors pin
    rng = np.random.default_rng(5)
    from kt_gguf_b200 import synth

    w = synth.random_blocks(rng, 42, 6, 1024)
    q8 = H.q2_0_to_q8_0(torch.from_numpy(w)).numpy()
    a, b = O.dequant(42, w, 1024), O.dequant(8, q8, 1024)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("native,type2", [("1", 42), ("0", 8), (None, 42)])
def test_q2_0_downs_native_or_repacked(monkeypatch, native, type2):
    # hot/kt_gguf_hot.py:180-190: Q2_0 downs stay 2-bit unless KT_GGUF_Q2_NATIVE=0
    if native is None:
        monkeypatch.delenv("KT_GGUF_Q2_NATIVE", raising=False)
    else:
        monkeypatch.setenv("KT_GGUF_Q2_NATIVE", native)
    H._readers["fake://q2"] = SimpleNamespace(types=lambda li: (12, 12, 42))
    kt = SimpleNamespace(num_gpu_experts=4, weight_path="fake://q2", layer_idx=0)
    m = H.KTGGUFHotExpertsMethod(kt, SimpleNamespace(moe_tp_rank=0, moe_tp_size=1))
    assert (m.type13, m.type2, m.q2_native) == (12, type2, native != "0")
    m.K, m.N = 2048, 512
    x = torch.zeros((4096, 2048), dtype=torch.bfloat16)
    # the prefill layer takes the four north-star types: a native Q2_0 layer stays on the GEMV
    assert m._use_prefill(x, 4096) == (type2 == 8 and H.PREFILL_ON_GPU)


def test_row_bytes_and_block_table():
    assert H._row_bytes(2048, 12) == 8 * 144 and H._row_bytes(512, 14) == 420 and H._row_bytes(512, 21) == 220
    with pytest.raises(ValueError):
        H._row_bytes(100, 12)
    assert H.MMVQ_TYPES == {2, 3, 6, 7, 8, 10, 11, 12, 13, 14, 16, 17, 18, 19, 20, 21, 22, 23, 29}
    assert all(H.BLOCK_INFO[t] == O.BLOCK[t] for t in H.MMVQ_TYPES | {42})
