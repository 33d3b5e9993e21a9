"""Decode-adaptive hot experts for the KT hybrid with GGUF experts — B200 implementation.

Drop-in for sglang.srt.layers.moe.kt_hot_cache (hot/kt_hot_cache.py): the GPU slots of
every layer follow the decode's own routing instead of a static map (KT_HOT_DYNAMIC=1).

Tables (int32 like the router's ids, on the GPU with host copies):
  log2slot [L, E]  slot holding logical expert e, or -1
  log2cpu  [L, E]  -1 for a resident expert, else the logical id itself
  counts   [L, E]  decayed route counts (float32)
route() is one kernel (kt_hot_route: both lookups and the count update, any number of
routes), so it can be captured in the decode graph; the swap policy runs between steps on
the host and changes the tables in place (push_tables). Residency is carried by the ids
alone: every expert is either in log2slot or in log2cpu, never both (check_tables).

Slot entries: a logical id, EMPTY (-1, filled first by the policy) or ABSENT (-2, a KV-lent
slot that does not exist now). Environment knobs as in the reference:
KT_HOT_INTERVAL, KT_HOT_SWAPS, KT_HOT_DECAY, KT_HOT_MARGIN, KT_HOT_SEED, KT_HOT_KV_LEND,
KT_HOT_KV_LEND_MAX, KT_HOT_LOG.
"""
import json
import os
import time
from typing import Dict, List, Optional

import torch

from . import kernels as _k

ENABLED = os.environ.get("KT_HOT_DYNAMIC") == "1"
INTERVAL = int(os.environ.get("KT_HOT_INTERVAL", "32"))
MAX_SWAPS = int(os.environ.get("KT_HOT_SWAPS", "8"))
DECAY = float(os.environ.get("KT_HOT_DECAY", "0.9"))
MARGIN = float(os.environ.get("KT_HOT_MARGIN", "1.5"))
SEED = os.environ.get("KT_HOT_SEED")
LOG_EVERY = int(os.environ.get("KT_HOT_LOG", "0"))
KV_LEND = os.environ.get("KT_HOT_KV_LEND", "0") == "1"
KV_LEND_MAX = int(os.environ.get("KT_HOT_KV_LEND_MAX", "64"))
FUSED_ROUTE = True  # route() is always the single native kernel here
EMPTY, ABSENT = -1, -2


def _log(msg):
    print(f"[kt-hot {time.strftime('%H:%M:%S')}] {msg}", flush=True)


class HotCache:
    def __init__(self, num_layers: int, num_experts: int, slots: int, device: torch.device, rank: int):
        self.L, self.E, self.N, self.device, self.rank = num_layers, num_experts, slots, device, rank
        self.log2slot_cpu = torch.full((num_layers, num_experts), -1, dtype=torch.int32)
        self.log2slot = self.log2slot_cpu.to(device, copy=True)
        self.log2cpu_cpu = torch.arange(num_experts, dtype=torch.int32).repeat(num_layers, 1)
        self.log2cpu = self.log2cpu_cpu.to(device, copy=True)
        self.counts = torch.zeros((num_layers, num_experts), dtype=torch.float32, device=device)
        self.S = slots + (KV_LEND_MAX if KV_LEND else 0)  # slot ids per layer (resident + lent)
        self.slot2log: List[List[int]] = [[EMPTY] * slots + [ABSENT] * (self.S - slots) for _ in range(num_layers)]
        self.lent_views: Dict[tuple, tuple] = {}
        if KV_LEND:
            # every B200 kernel reads slots through the pointer tables (kt_gguf_moe_multi.reads_table),
            # so the base tables only mirror the full ones for callers that ask for them
            self.log2slot_base_cpu = self.log2slot_cpu.clone()
            self.log2cpu_base_cpu = self.log2cpu_cpu.clone()
            self.log2slot_base = self.log2slot.clone()
            self.log2cpu_base = self.log2cpu.clone()
        self.layers: Dict[int, tuple] = {}  # layer_idx -> (hot method, FusedMoE layer)
        self._mirrors: Dict[tuple, Optional[torch.Tensor]] = {}
        self._counts_host = torch.zeros((num_layers, num_experts), dtype=torch.float32)
        if torch.cuda.is_available():
            self._counts_host = self._counts_host.pin_memory()
        self._counts_event = None
        self._own_banks: Dict[int, list] = {}
        self.ready = False
        self.step = self.rounds = self.swaps = self.bytes = 0
        self.swap_s = 0.0

    # -- graph side ----------------------------------------------------------

    def route(self, layer_idx: int, ids: torch.Tensor):
        """ids: logical [T, k] int32 (>= 0). Returns (slot ids with -1 for experts on the CPU,
        logical ids with -1 for the resident ones) and counts each route. One kernel."""
        slot_tab, cpu_tab = self.log2slot, self.log2cpu
        if KV_LEND:
            from . import kt_gguf_moe_multi as _multi

            if not _multi.reads_table(ids.shape[0]):
                # a kernel that addresses base + slot * stride: lent residents go to the CPU
                slot_tab, cpu_tab = self.log2slot_base, self.log2cpu_base
        return _k.hot_route(ids.to(torch.int32), slot_tab[layer_idx], cpu_tab[layer_idx], self.counts[layer_idx])

    def push_tables(self) -> None:
        """The host tables to the GPU on the current stream."""
        self.log2slot.copy_(self.log2slot_cpu, non_blocking=True)
        self.log2cpu.copy_(self.log2cpu_cpu, non_blocking=True)
        if KV_LEND:
            self.log2slot_base.copy_(self.log2slot_base_cpu, non_blocking=True)
            self.log2cpu_base.copy_(self.log2cpu_base_cpu, non_blocking=True)

    # -- filling -------------------------------------------------------------

    def _bank(self, layer_idx: int):
        """This rank's slice of every expert of the layer (gate, up, down) in pinned host
        memory, built once from the hot method's GGUF reader."""
        b = self._own_banks.get(layer_idx)
        if b is not None:
            return b
        method, _layer = self.layers[layer_idx]
        rd, N, r = method.reader, method.N, method.rank
        experts = torch.arange(rd.E)
        try:  # banks in physical order when a placement map renumbers the experts
            from sglang.srt.eplb.expert_location_dispatch import get_global_expert_location_metadata

            meta = get_global_expert_location_metadata()
            if meta is not None:
                experts = meta.physical_to_logical_map_cpu[layer_idx].to(torch.int64)
        except ImportError:
            pass
        banks = []
        for proj in ("gate", "up", "down"):
            v = rd.slice(layer_idx, proj, N, r, experts).reshape(rd.E, -1)
            h = torch.empty(v.shape, dtype=torch.uint8, pin_memory=torch.cuda.is_available())
            h.copy_(v)
            banks.append(h)
        self._own_banks[layer_idx] = banks
        return banks

    def fill(self, layer_idx: int, slot: int, logical: int) -> None:
        """Copies an expert's gate/up/down slices from the banks into a slot."""
        method, layer = self.layers[layer_idx]
        gate, up, down = self._bank(layer_idx)
        N = method.N
        if slot >= self.N:
            v13, v2 = self.lent_views[(layer_idx, slot)]
        else:
            v13, v2 = layer.w13_qweight.data[slot], layer.w2_qweight.data[slot]
        d = down[logical].view(v2.shape[0], -1)
        if method.types[2] != method.type2:  # Q2_0 downs are kept as exact Q8_0 repacks
            from .kt_gguf_hot import q2_0_to_q8_0

            d = q2_0_to_q8_0(d)
        v13[:N].copy_(gate[logical].view(N, -1), non_blocking=True)
        v13[N:].copy_(up[logical].view(N, -1), non_blocking=True)
        v2.copy_(d, non_blocking=True)
        self.bytes += gate[logical].numel() + up[logical].numel() + d.numel()

    def _set(self, layer_idx: int, slot: int, logical: int) -> None:
        """Slot <- logical (>= 0), or EMPTY / ABSENT; the previous resident goes back to the CPU
        tables."""
        old = self.slot2log[layer_idx][slot]
        if old >= 0:
            self.log2slot_cpu[layer_idx, old] = -1
            self.log2cpu_cpu[layer_idx, old] = old
            if KV_LEND and slot < self.N:
                self.log2slot_base_cpu[layer_idx, old] = -1
                self.log2cpu_base_cpu[layer_idx, old] = old
        self.slot2log[layer_idx][slot] = logical
        if logical < 0:
            return
        self.log2slot_cpu[layer_idx, logical] = slot
        self.log2cpu_cpu[layer_idx, logical] = -1
        if KV_LEND and slot < self.N:
            self.log2slot_base_cpu[layer_idx, logical] = slot
            self.log2cpu_base_cpu[layer_idx, logical] = -1

    def check_tables(self) -> str:
        """'' if every expert of every layer is exactly once on a slot that holds it or on the
        CPU, in host and device tables; else the first violation."""
        pairs = [("full", self.log2slot_cpu, self.log2cpu_cpu, self.log2slot, self.log2cpu, False)]
        if KV_LEND:
            pairs.append(("base", self.log2slot_base_cpu, self.log2cpu_base_cpu, self.log2slot_base, self.log2cpu_base,
                          True))
        ids = torch.arange(self.E, dtype=torch.int32)
        for name, s_cpu, c_cpu, s_dev, c_dev, base in pairs:
            if not torch.equal(s_dev.cpu(), s_cpu) or not torch.equal(c_dev.cpu(), c_cpu):
                return f"{name}: device tables differ from the host's"
            if not bool(((s_cpu >= 0) ^ (c_cpu >= 0)).all()):
                return f"{name}: an expert both or neither on a slot and on the CPU"
            if not bool(((c_cpu < 0) | (c_cpu == ids)).all()):
                return f"{name}: CPU id is not the logical id"
            for li in range(self.L):
                for e in (s_cpu[li] >= 0).nonzero().flatten().tolist():
                    sl = int(s_cpu[li, e])
                    if self.slot2log[li][sl] != e or (base and sl >= self.N):
                        return f"{name}: layer {li} expert {e} -> slot {sl} holding {self.slot2log[li][sl]}"
                for sl, e in enumerate(self.slot2log[li]):
                    if e >= 0 and int(self.log2slot_cpu[li, e]) != sl:
                        return f"{name}: layer {li} slot {sl} holds {e} but the table says {int(self.log2slot_cpu[li, e])}"
        return ""

    # -- lent slots -------------------------------------------------------------

    def lend_slot(self, layer_idx: int, slot: int, v13: torch.Tensor, v2: torch.Tensor) -> None:
        if self.slot2log[layer_idx][slot] != ABSENT:
            raise RuntimeError(f"slot {slot} of layer {layer_idx} already exists")
        self.lent_views[(layer_idx, slot)] = (v13, v2)
        self.slot2log[layer_idx][slot] = EMPTY

    def take_back_slot(self, layer_idx: int, slot: int) -> int:
        """The slot's expert goes back to the CPU (host tables; push_tables before the next
        forward). Returns the expert it held or -1."""
        old = self.slot2log[layer_idx][slot]
        if old == ABSENT:
            raise RuntimeError(f"slot {slot} of layer {layer_idx} is not lent")
        self._set(layer_idx, slot, ABSENT)
        del self.lent_views[(layer_idx, slot)]
        return old

    def fill_empty(self, counts: torch.Tensor, seed_rank: Optional[torch.Tensor] = None) -> int:
        """Every EMPTY slot gets the hottest non-resident expert of its layer (ties broken by the
        seed map's order). Host tables only."""
        n = 0
        for li in sorted(self.layers):
            empty = [s for s, e in enumerate(self.slot2log[li]) if e == EMPTY]
            if not empty:
                continue
            score = counts[li].double().clone()
            if seed_rank is not None:
                score += (self.E - seed_rank[li].double()) / (self.E + 1) * 1e-3
            res = [e for e in self.slot2log[li] if e >= 0]
            if res:
                score[torch.tensor(res)] = float("-inf")
            for s, c in zip(empty, torch.topk(score, len(empty)).indices.tolist()):
                self._set(li, s, c)
                self.fill(li, s, c)
                n += 1
        return n

    def seed(self, placement: Optional[str]) -> None:
        """Initial residents: the placement map's first N per layer, or logical 0..N-1."""
        p2l = json.load(open(placement))["physical_to_logical_map"] if placement else None
        for li in sorted(self.layers):
            for s in range(self.N):
                e = int(p2l[li][s]) if p2l else s
                self._set(li, s, e)
                if p2l and e != s:
                    self.fill(li, s, e)
        self.push_tables()
        if torch.cuda.is_available():
            torch.cuda.current_stream(self.device).synchronize()
        self.ready = True
        self.bytes = 0

    # -- policy, between steps --------------------------------------------------

    def plan_swaps(self, counts: torch.Tensor):
        """Pairs (layer, slot, expert) to swap in: per layer the coldest residents give way to
        the hottest non-residents when candidate > MARGIN * resident, at most MAX_SWAPS, in
        order of the coldest slot first (EMPTY slots score -1, ABSENT ones never swap)."""
        res = torch.tensor(self.slot2log)  # [L, S]
        score_res = counts.gather(1, res.clamp(min=0))
        score_res = torch.where(res == EMPTY, torch.full_like(score_res, -1.0), score_res)
        score_res = torch.where(res == ABSENT, torch.full_like(score_res, float("inf")), score_res)
        nonres = torch.ones((counts.shape[0], counts.shape[1] + 1), dtype=torch.bool)
        nonres.scatter_(1, torch.where(res >= 0, res, torch.full_like(res, counts.shape[1])), False)
        nonres = nonres[:, :-1]
        k = min(MAX_SWAPS, counts.shape[1], res.shape[1])
        cand_score, cand_idx = torch.topk(torch.where(nonres, counts, torch.full_like(counts, -1.0)), k, dim=1)
        order = torch.argsort(score_res, dim=1)[:, :k]  # coldest slots first
        rs = score_res.gather(1, order)
        do = ((cand_score > 0) & (cand_score > MARGIN * rs)).to(torch.int64).cumprod(1).bool()
        return [(li, int(order[li, j]), int(cand_idx[li, j])) for li, j in do.nonzero().tolist()]

    def before_forward(self, forward_batch) -> None:
        mode = forward_batch.forward_mode
        if not self.ready or not (mode.is_decode() or mode.is_target_verify()):
            return
        self.step += 1
        if self.step % INTERVAL:
            return
        t0 = time.time()
        # the counts come back through a pinned buffer one round late, so the policy never
        # waits for the step in flight
        if self._counts_event is not None and not self._counts_event.query():
            return
        counts = self._counts_host.clone() if self._counts_event is not None else None
        self._counts_host.copy_(self.counts, non_blocking=True)
        self.counts.mul_(DECAY)
        if self._counts_event is None:
            self._counts_event = torch.cuda.Event()
        self._counts_event.record(torch.cuda.current_stream(self.device))
        if counts is None:
            return
        swaps = 0
        for li, s, c in self.plan_swaps(counts):
            if li not in self.layers:
                continue
            self._set(li, s, c)
            self.fill(li, s, c)
            swaps += 1
        if swaps:
            self.push_tables()
        self.rounds += 1
        self.swaps += swaps
        self.swap_s += time.time() - t0
        if self.rounds == 1 or (LOG_EVERY and self.rounds % LOG_EVERY == 0) or self.rounds % 64 == 0:
            resident = sum(float(counts[li][torch.tensor([e for e in self.slot2log[li] if e >= 0], dtype=torch.long)].sum())
                           for li in self.layers)
            _log(f"rank {self.rank}: round {self.rounds} (step {self.step}): {swaps} swaps this round, "
                 f"{self.swaps} total, {self.bytes / 1e9:.2f} GB, {self.swap_s * 1e3 / self.rounds:.1f} ms/round; "
                 f"GPU share of recent routes {resident / max(float(counts.sum()), 1):.3f}")


_cache: Optional[HotCache] = None


def register(method, layer) -> Optional[HotCache]:
    """Called by the KT wrapper on its first decode apply of each layer; the cache is built on
    the first call and seeded once every layer is known."""
    global _cache
    if not ENABLED:
        return None
    kt = method.kt_config
    if _cache is None:
        if kt.num_gpu_experts <= 0:
            raise RuntimeError("KT_HOT_DYNAMIC=1 needs --kt-num-gpu-experts > 0")
        _cache = HotCache(kt.num_layers, method.global_num_experts, kt.num_gpu_experts, layer.w13_qweight.device,
                          method.tp_rank)
    c = _cache
    if kt.layer_idx not in c.layers:
        c.layers[kt.layer_idx] = (method.gpu_method, layer)
        if len(c.layers) == kt.num_layers:
            c.seed(SEED)
    return c if c.ready else None


def before_forward(forward_batch) -> None:
    if _cache is not None:
        _cache.before_forward(forward_batch)
