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


class CountingReader(FakeReader):
    def __init__(self):
        super().__init__()
        self.calls = 0

    def slice(self, li, proj, N, rank, experts):
        self.calls += 1
        return super().slice(li, proj, N, rank, experts)


def test_own_bank_is_built_once_per_layer(monkeypatch):
    c = make_cache(monkeypatch=monkeypatch)
    rd = CountingReader()
    for li in range(L):
        c.layers[li][0].reader = rd
    c.seed(None)
    for e in (9, 10, 11):
        c._set(0, 1, e)
        c.fill(0, 1, e)
        assert slot_bytes(c, 0, 1) == expect_bytes(0, e)
    assert rd.calls == 3  # gate, up, down of layer 0, once
    assert c._bank(0).source == "own"


def test_banks_shared_with_the_streamer(monkeypatch):
    # with the GGUF streamer loaded, fills read its pinned banks (one copy of every expert for
    # both); KT_HOT_BANKS=own keeps the cache's own
    from kt_gguf_b200 import kt_stream_prefill_gguf as G

    class FakeStreamer:
        def _bank(self, li):
            w13 = torch.full((E, 2 * N_INTER * ROWB13), 200 + li, dtype=torch.uint8)
            w2 = torch.full((E, 2 * N_INTER * ROWB2), 210 + li, dtype=torch.uint8)
            return [w13, w2]

    monkeypatch.setattr(G, "_instance", FakeStreamer())
    c = make_cache(monkeypatch=monkeypatch)
    rd = CountingReader()
    c.layers[1][0].reader = rd
    c.seed(None)
    c._set(1, 2, 12)
    c.fill(1, 2, 12)
    assert slot_bytes(c, 1, 2) == (201, 201, 211) and rd.calls == 0
    assert c._bank(1).source == "streamer"
    monkeypatch.setattr(C, "OWN_BANKS", "own")
    c2 = make_cache(monkeypatch=monkeypatch)
    c2.seed(None)
    c2._set(1, 2, 12)
    c2.fill(1, 2, 12)
    assert slot_bytes(c2, 1, 2) == expect_bytes(1, 12)


def test_fill_writes_the_lend_mirror(monkeypatch):
    # a resident slot's new expert also goes to the host mirror the weight return restores from
    # (hot/kt_hot_cache.py:207-226, 264-270); lent slots have no mirror
    c = make_cache(kv_lend=True, monkeypatch=monkeypatch)
    c.seed(None)
    _m, layer = c.layers[0]
    m13, m2 = torch.zeros_like(layer.w13_qweight), torch.zeros_like(layer.w2_qweight)
    c.register_mirror(layer.w13_qweight, m13)
    c.register_mirror(layer.w2_qweight, m2)
    with pytest.raises(ValueError):
        c.register_mirror(layer.w2_qweight, torch.zeros(3, dtype=torch.uint8))
    c._set(0, 3, 14)
    c.fill(0, 3, 14)
    g, u, d = expect_bytes(0, 14)
    assert bool((m13[3, :N_INTER] == g).all() and (m13[3, N_INTER:] == u).all() and (m2[3] == d).all())
    assert bool((m13[:3] == 0).all())
    v13 = torch.zeros((2 * N_INTER, ROWB13), dtype=torch.uint8)
    v2 = torch.zeros((2 * N_INTER, ROWB2), dtype=torch.uint8)
    c.lend_slot(0, NS, v13, v2)
    before = m13.clone()
    c._set(0, NS, 15)
    c.fill(0, NS, 15)
    assert torch.equal(m13, before) and slot_bytes(c, 0, NS) == expect_bytes(0, 15)


def test_q2_0_down_bank_is_repacked_once(monkeypatch):
    # a layer whose Q2_0 downs are kept as their Q8_0 repack: the whole down bank is repacked
    # once (hot/kt_hot_cache.py:228-243), each fill copies from it
    rng = np.random.default_rng(1)
    n_blk = 4  # Q2_0 blocks per down row (256 values)
    down_raw = rng.integers(0, 256, size=(E, 2 * N_INTER, n_blk * 18), dtype=np.uint8)
    down_raw.reshape(-1, 18)[:, 1] &= 0x3B  # finite fp16 scales

    class Q2Reader(FakeReader):
        def slice(self, li, proj, N, rank, experts):
            if proj != "down":
                return super().slice(li, proj, N, rank, experts)
            return torch.from_numpy(down_raw[experts.numpy()])

    monkeypatch.setattr(C, "KV_LEND", False)
    c = C.HotCache(1, E, NS, torch.device("cpu"), 0)
    method = SimpleNamespace(reader=Q2Reader(), N=N_INTER, rank=0, types=(12, 12, 42), type2=8)
    layer = SimpleNamespace(w13_qweight=torch.zeros((NS, 2 * N_INTER, ROWB13), dtype=torch.uint8),
                            w2_qweight=torch.zeros((NS, 2 * N_INTER, n_blk * 68), dtype=torch.uint8))
    c.layers[0] = (method, layer)
    c.seed(None)
    for s, e in ((0, 7), (1, 9)):
        c._set(0, s, e)
        c.fill(0, s, e)
        want = H.q2_0_to_q8_0(torch.from_numpy(down_raw[e]))
        assert torch.equal(layer.w2_qweight[s], want)
    assert list(c._q8_down) == [0]


class _Mode:
    def __init__(self, decode):
        self.decode = decode

    def is_decode(self):
        return self.decode

    def is_target_verify(self):
        return False


def test_before_forward_uses_counts_one_round_late(monkeypatch):
    monkeypatch.setattr(C, "INTERVAL", 2)
    monkeypatch.setattr(C, "MAX_SWAPS", 2)
    monkeypatch.setattr(C, "DECAY", 0.5)
    c = make_cache(monkeypatch=monkeypatch)
    c.seed(None)
    batch = SimpleNamespace(forward_mode=_Mode(True))
    prefill = SimpleNamespace(forward_mode=_Mode(False))
    c.counts[0, 12] = 40.0  # hot non-resident expert of layer 0
    c.counts[0, :NS] = torch.tensor([9.0, 1.0, 9.0, 9.0])
    c.before_forward(prefill)  # prefill steps do not count
    c.before_forward(batch)    # step 1: not a policy step
    assert c.step == 1 and c.rounds == 0
    c.before_forward(batch)    # step 2: the first round only starts the copy of the counts
    assert c.rounds == 0 and float(c.counts[0, 12]) == 20.0  # decayed after the copy
    assert c.slot2log[0][:NS] == [0, 1, 2, 3]
    c.before_forward(batch)
    c.before_forward(batch)    # step 4: the counts of round 1 (40 vs 1) swap 12 into slot 1
    assert c.rounds == 1 and c.swaps == 1
    assert c.slot2log[0][1] == 12 and int(c.log2slot[0, 12]) == 1 and int(c.log2cpu[0, 1]) == 1
    assert c.check_tables() == "" and slot_bytes(c, 0, 1) == expect_bytes(0, 12)


def test_plan_swaps_function_matches_the_method(monkeypatch):
    c = make_cache(monkeypatch=monkeypatch)
    c.seed(None)
    rng = np.random.default_rng(4)
    counts = rng.integers(0, 6, size=(L, E)).astype(np.float32)
    assert C.plan_swaps(counts, c.slot2log, C.MAX_SWAPS, C.MARGIN) == c.plan_swaps(torch.from_numpy(counts))
