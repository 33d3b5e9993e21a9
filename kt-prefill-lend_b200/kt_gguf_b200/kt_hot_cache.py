"""Decode-adaptive hot experts for the KT hybrid with GGUF experts — B200 implementation.

Drop-in for sglang.srt.layers.moe.kt_hot_cache (hot/kt_hot_cache.py): with KT_HOT_DYNAMIC=1 the
GPU slots of every layer follow the decode's own routing instead of a static map. The public
surface is the reference's (HotCache with route / push_tables / fill / fill_empty / seed /
check_tables / lend_slot / take_back_slot / before_forward, its attributes log2slot, log2cpu,
counts, slot2log, lent_views, layers, S, N; module functions register and before_forward; the
KT_HOT_* environment knobs); the implementation is this package's own:

- Tables. Residency lives in one int32 block [kinds, L, E] on the host (pageable, so a push
  never races a later edit) and one on the GPU, pushed with a single copy: kind 0 the slot of
  each logical expert (-1: not resident), kind 1 the id the CPU computes (-1: resident), and
  with KV_LEND kinds 2 and 3 the same for the "base" view in which lent slots do not exist.
  log2slot / log2cpu (and *_cpu, *_base) are views into the blocks. route() is one kernel
  (kt_hot_route) at any size, so it is captured with the decode graph.
- Slots. slot2log[l][s] is the slot's logical expert, EMPTY (-1, filled first) or ABSENT (-2, a
  lent slot that does not exist now). Every table edit goes through _set, which moves one
  expert out of and one into a slot, so an expert is always exactly once on a slot or on the
  CPU (check_tables verifies it, host and device).
- Expert bytes. A swap copies the expert from a pinned bank whose rows already have the slot
  layout (gate rows then up rows, then the down matrix): two copies per fill. The bank is the
  GGUF streamer's (kt_stream_prefill_gguf, one pinned copy of every expert serves both) unless
  KT_HOT_BANKS=own or the streamer cannot serve the layer; otherwise the cache builds its own
  from the hot method's reader, once per layer. Layers whose Q2_0 down is kept as its exact
  Q8_0 repack get a repacked down bank, built once per layer.
- Lend mirror. A resident slot's bytes also go to the host mirror of its parameter, so a
  weight return after a prefill restores the swapped-in expert, not the old one: mirrors
  registered with register_mirror(param, host), or found in the reference's kt_lend state.
  Lent slots (KV pages) have none; they are given back before every streamed prefill.
- Policy, between decode steps (before_forward): every KT_HOT_INTERVAL decode or target-verify
  steps, the route counts come back through a pinned buffer one round late (the policy never
  waits for the step in flight), decay by KT_HOT_DECAY, and per layer the coldest slots give
  way to the hottest non-resident experts while candidate > KT_HOT_MARGIN * resident, at most
  KT_HOT_SWAPS per layer, stopping at the first pair that fails (plan_swaps).

KT_HOT_SEED=<placement json> seeds the slots from physical_to_logical_map (first N per layer);
without it slot s starts with logical expert s. KT_HOT_KV_LEND=1 adds up to KT_HOT_KV_LEND_MAX
lent slots per layer (ids N..S-1).
"""
import json
import os
import time
from typing import Dict, List, Optional, Tuple

import numpy as np
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
OWN_BANKS = os.environ.get("KT_HOT_BANKS", "auto")  # "own": never share the streamer's banks
FUSED_ROUTE = True  # route() is always the single native kernel here
EMPTY, ABSENT = -1, -2

# kinds of the residency block
_SLOT, _CPU, _SLOT_BASE, _CPU_BASE = 0, 1, 2, 3


def _log(msg):
    print(f"[kt-hot {time.strftime('%H:%M:%S')}] {msg}", flush=True)


class ExpertBank:
    """Pinned bytes of every expert of one layer in slot layout (physical expert order):
    w13 [E, 2N * row_bytes13] (gate rows, then up rows) and w2 [E, K * row_bytes2]."""

    def __init__(self, w13: torch.Tensor, w2: torch.Tensor, source: str):
        if w13.shape[0] != w2.shape[0]:
            raise ValueError("gate/up and down banks disagree on the expert count")
        self.w13, self.w2, self.source = w13, w2, source

    @property
    def nbytes(self) -> int:
        return self.w13.numel() + self.w2.numel()


def plan_swaps(counts: np.ndarray, slot2log: List[List[int]], max_swaps: int, margin: float,
               layers=None) -> List[Tuple[int, int, int]]:
    """Swaps (layer, slot, expert) for one policy round. Per layer, slots are taken coldest
    first (an EMPTY slot scores -1, an ABSENT one never swaps) and non-resident experts hottest
    first, both at most max_swaps; the j-th pair swaps while the candidate's count is positive
    and above margin times the slot's, and the first pair that fails ends the layer's list."""
    counts = np.asarray(counts, dtype=np.float64)
    n_layers, n_exp = counts.shape
    k = min(max_swaps, n_exp, len(slot2log[0]) if slot2log else 0)
    out = []
    for li in range(n_layers) if layers is None else sorted(layers):
        held = np.asarray(slot2log[li], dtype=np.int64)
        score = np.where(held >= 0, counts[li][np.clip(held, 0, None)], 0.0)
        score = np.where(held == EMPTY, -1.0, score)
        score = np.where(held == ABSENT, np.inf, score)
        slots = np.argsort(score, kind="stable")[:k]
        free = counts[li].copy()
        free[held[held >= 0]] = -1.0  # residents are not candidates
        cands = np.argsort(-free, kind="stable")[:k]
        for s, e in zip(slots.tolist(), cands.tolist()):
            c, r = free[e], score[s]
            if not (c > 0 and c > margin * r):
                break
            out.append((li, int(s), int(e)))
    return out


class HotCache:
    def __init__(self, num_layers: int, num_experts: int, slots: int, device: torch.device, rank: int):
        self.L, self.E, self.N, self.device, self.rank = num_layers, num_experts, slots, device, rank
        self.S = slots + (KV_LEND_MAX if KV_LEND else 0)  # slot ids per layer: resident, then lent
        kinds = 4 if KV_LEND else 2
        tab = torch.empty((kinds, num_layers, num_experts), dtype=torch.int32)
        tab[_SLOT::2] = -1
        tab[_CPU::2] = torch.arange(num_experts, dtype=torch.int32)
        self._tab_host = tab
        self._tab_dev = tab.to(device, copy=True)
        self.log2slot_cpu, self.log2cpu_cpu = tab[_SLOT], tab[_CPU]
        self.log2slot, self.log2cpu = self._tab_dev[_SLOT], self._tab_dev[_CPU]
        if KV_LEND:
            self.log2slot_base_cpu, self.log2cpu_base_cpu = tab[_SLOT_BASE], tab[_CPU_BASE]
            self.log2slot_base, self.log2cpu_base = self._tab_dev[_SLOT_BASE], self._tab_dev[_CPU_BASE]
        self.counts = torch.zeros((num_layers, num_experts), dtype=torch.float32, device=device)
        self.slot2log: List[List[int]] = [[EMPTY] * slots + [ABSENT] * (self.S - slots) for _ in range(num_layers)]
        self.lent_views: Dict[Tuple[int, int], Tuple[torch.Tensor, torch.Tensor]] = {}
        self.layers: Dict[int, tuple] = {}  # layer_idx -> (hot method, FusedMoE layer)
        self.mirrors: Dict[int, torch.Tensor] = {}  # parameter data_ptr -> its host mirror
        self._banks: Dict[int, ExpertBank] = {}
        self._q8_down: Dict[int, torch.Tensor] = {}
        self._round_counts = None  # (pinned host buffer, event of its copy) of the previous round
        self.ready = False
        self.step = self.rounds = self.swaps = self.bytes = 0
        self.swap_s = 0.0

    # -- graph side ----------------------------------------------------------

    def route(self, layer_idx: int, ids: torch.Tensor):
        """ids: logical [T, k] int32 (>= 0). Returns (slot ids with -1 for experts on the CPU,
        logical ids with -1 for the resident ones) and counts each route. One kernel."""
        kind = (_SLOT, _CPU)
        if KV_LEND:
            from . import kt_gguf_moe_multi as _multi

            if not _multi.reads_table(ids.shape[0]):
                kind = (_SLOT_BASE, _CPU_BASE)  # a kernel without slot tables: lent residents on the CPU
        return _k.hot_route(ids.to(torch.int32), self._tab_dev[kind[0], layer_idx], self._tab_dev[kind[1], layer_idx],
                            self.counts[layer_idx])

    def push_tables(self) -> None:
        """Every table to the GPU, one copy on the current stream."""
        self._tab_dev.copy_(self._tab_host, non_blocking=True)

    # -- residency -------------------------------------------------------------

    def _kinds(self, slot: int):
        """table pairs a slot appears in: the full view always, the base view only for resident
        (not lent) slots"""
        if KV_LEND and slot < self.N:
            return ((_SLOT, _CPU), (_SLOT_BASE, _CPU_BASE))
        return ((_SLOT, _CPU),)

    def _set(self, layer_idx: int, slot: int, logical: int) -> None:
        """Slot <- logical (>= 0), EMPTY or ABSENT; the expert it held goes back to the CPU."""
        t = self._tab_host
        prev = self.slot2log[layer_idx][slot]
        for ks, kc in self._kinds(slot):
            if prev >= 0:
                t[ks, layer_idx, prev], t[kc, layer_idx, prev] = -1, prev
            if logical >= 0:
                t[ks, layer_idx, logical], t[kc, layer_idx, logical] = slot, -1
        self.slot2log[layer_idx][slot] = logical

    def check_tables(self) -> str:
        """'' if every expert of every layer is exactly once on a slot that holds it or on the
        CPU, in host and device tables; else the first violation found."""
        if not torch.equal(self._tab_dev.cpu(), self._tab_host):
            return "device tables differ from the host's"
        ids = torch.arange(self.E, dtype=torch.int32)
        views = [("full", _SLOT, _CPU)] + ([("base", _SLOT_BASE, _CPU_BASE)] if KV_LEND else [])
        for name, ks, kc in views:
            s_tab, c_tab = self._tab_host[ks], self._tab_host[kc]
            on_slot, on_cpu = s_tab >= 0, c_tab >= 0
            if bool((on_slot == on_cpu).any()):
                li, e = (on_slot == on_cpu).nonzero()[0].tolist()
                return f"{name}: layer {li} expert {e} is on both or neither of a slot and the CPU"
            if bool((on_cpu & (c_tab != ids)).any()):
                return f"{name}: a CPU id is not the expert's own id"
            for li in range(self.L):
                held = self.slot2log[li]
                for e in on_slot[li].nonzero().flatten().tolist():
                    s = int(s_tab[li, e])
                    if held[s] != e:
                        return f"{name}: layer {li} expert {e} points at slot {s}, which holds {held[s]}"
                    if name == "base" and s >= self.N:
                        return f"base: layer {li} expert {e} on lent slot {s}"
                for s, e in enumerate(held):
                    if e >= 0 and int(self._tab_host[_SLOT, li, e]) != s:
                        return f"{name}: layer {li} slot {s} holds {e}, the table says slot {int(self._tab_host[_SLOT, li, e])}"
        return ""

    # -- expert bytes ----------------------------------------------------------

    def _bank(self, layer_idx: int) -> ExpertBank:
        b = self._banks.get(layer_idx)
        if b is None:
            b = self._streamer_bank(layer_idx) if OWN_BANKS != "own" else None
            if b is None:
                b = self._own_bank(layer_idx)
            self._banks[layer_idx] = b
        return b

    def _streamer_bank(self, layer_idx: int) -> Optional[ExpertBank]:
        """The GGUF streamer's pinned bank of the layer, when the streamer is loaded and can hold
        this layer's types (its banks have the slot layout too)."""
        from . import kt_stream_prefill_gguf as G

        inst = G._instance
        if inst is None:
            return None
        try:
            w13, w2 = inst._bank(layer_idx)
        except RuntimeError:  # a type the streamer's GEMMs do not take
            return None
        return ExpertBank(w13, w2, "streamer")

    def _own_bank(self, layer_idx: int) -> ExpertBank:
        """This rank's slice of every expert of the layer, from the hot method's GGUF reader."""
        t0 = time.time()
        method, _layer = self.layers[layer_idx]
        rd, n = method.reader, method.N
        order = _physical_order(layer_idx, rd.E)
        pin = torch.cuda.is_available()
        parts = [rd.slice(layer_idx, p, n, method.rank, order).reshape(rd.E, -1) for p in ("gate", "up", "down")]
        w13 = torch.empty((rd.E, parts[0].shape[1] + parts[1].shape[1]), dtype=torch.uint8, pin_memory=pin)
        torch.cat(parts[:2], dim=1, out=w13)
        w2 = torch.empty(parts[2].shape, dtype=torch.uint8, pin_memory=pin)
        w2.copy_(parts[2])
        bank = ExpertBank(w13, w2, "own")
        if layer_idx == min(self.layers):
            _log(f"rank {self.rank}: layer {layer_idx} expert bank {bank.nbytes / 1e9:.2f} GB pinned in "
                 f"{time.time() - t0:.1f} s")
        return bank

    def _down_bytes(self, layer_idx: int, method, bank: ExpertBank) -> torch.Tensor:
        """The down matrices a slot is filled from: the bank's, or for a layer whose Q2_0 down is
        kept as its Q8_0 repack, that repack of the whole layer (built once, pinned)."""
        if method.types[2] == method.type2:
            return bank.w2
        q8 = self._q8_down.get(layer_idx)
        if q8 is None:
            from .kt_gguf_hot import q2_0_to_q8_0

            t0 = time.time()
            q8 = q2_0_to_q8_0(bank.w2)
            if torch.cuda.is_available():
                q8 = q8.pin_memory()
            self._q8_down[layer_idx] = q8
            _log(f"rank {self.rank}: layer {layer_idx} Q2_0 downs repacked to Q8_0 once for the slots "
                 f"({q8.numel() / 1e9:.2f} GB, {time.time() - t0:.1f} s)")
        return q8

    def register_mirror(self, param: torch.Tensor, host: torch.Tensor) -> None:
        """host (same shape and dtype) is the host copy the weight return restores `param` from;
        fills of resident slots write it too."""
        if tuple(host.shape) != tuple(param.shape) or host.dtype != param.dtype or host.is_cuda:
            raise ValueError("a mirror is a host tensor of the parameter's shape and dtype")
        self.mirrors[param.data_ptr()] = host

    def _mirror(self, param: torch.Tensor) -> Optional[torch.Tensor]:
        m = self.mirrors.get(param.data_ptr())
        if m is None:
            m = _reference_lend_mirror(param)
            if m is not None:
                self.mirrors[param.data_ptr()] = m
        return m

    def fill(self, layer_idx: int, slot: int, logical: int) -> None:
        """Copies an expert's bytes into a slot (a lent slot's KV-page views, or the layer's
        parameters and their host mirrors)."""
        method, layer = self.layers[layer_idx]
        bank = self._bank(layer_idx)
        src13 = bank.w13[logical]
        src2 = self._down_bytes(layer_idx, method, bank)[logical]
        lent = slot >= self.N
        if lent:
            dst13, dst2 = self.lent_views[(layer_idx, slot)]
        else:
            dst13, dst2 = layer.w13_qweight.data[slot], layer.w2_qweight.data[slot]
        dst13.copy_(src13.view(dst13.shape), non_blocking=True)
        dst2.copy_(src2.view(dst2.shape), non_blocking=True)
        if not lent:
            for param, src in ((layer.w13_qweight, src13), (layer.w2_qweight, src2)):
                m = self._mirror(param)
                if m is not None:
                    m[slot].copy_(src.view(m[slot].shape))
        self.bytes += src13.numel() + src2.numel()

    # -- lent slots ------------------------------------------------------------

    def lend_slot(self, layer_idx: int, slot: int, v13: torch.Tensor, v2: torch.Tensor) -> None:
        if self.slot2log[layer_idx][slot] != ABSENT:
            raise RuntimeError(f"layer {layer_idx}: slot {slot} exists already")
        self.lent_views[(layer_idx, slot)] = (v13, v2)
        self.slot2log[layer_idx][slot] = EMPTY

    def take_back_slot(self, layer_idx: int, slot: int) -> int:
        """The lent slot stops existing; its expert goes back to the CPU (host tables: push them
        before the next forward). Returns that expert, or -1."""
        held = self.slot2log[layer_idx][slot]
        if held == ABSENT:
            raise RuntimeError(f"layer {layer_idx}: slot {slot} is not lent")
        self._set(layer_idx, slot, ABSENT)
        del self.lent_views[(layer_idx, slot)]
        return held

    # -- seeding and filling -----------------------------------------------------

    def fill_empty(self, counts: torch.Tensor, seed_rank: Optional[torch.Tensor] = None) -> int:
        """Each EMPTY slot gets the hottest expert of its layer not resident yet (counts [L, E]
        on the host; equal counts go by the seed map's order). Host tables only."""
        done = 0
        c = np.asarray(counts, dtype=np.float64)
        for li in sorted(self.layers):
            empty = [s for s, e in enumerate(self.slot2log[li]) if e == EMPTY]
            if not empty:
                continue
            key = c[li].copy()
            if seed_rank is not None:
                # a tie-break far below one route: earlier in the seed map is hotter
                key += (self.E - np.asarray(seed_rank[li], dtype=np.float64)) / (self.E + 1) * 1e-3
            key[[e for e in self.slot2log[li] if e >= 0]] = -np.inf
            for s, e in zip(empty, np.argsort(-key, kind="stable")[:len(empty)].tolist()):
                self._set(li, s, e)
                self.fill(li, s, e)
                done += 1
        return done

    def seed(self, placement: Optional[str]) -> None:
        """Initial residents: the placement map's first N experts per layer, or logical 0..N-1
        (what the hot method loaded); slots whose expert differs from the loaded one are filled."""
        t0 = time.time()
        p2l = None
        if placement:
            with open(placement) as f:
                p2l = json.load(f)["physical_to_logical_map"]
        for li in sorted(self.layers):
            for s in range(self.N):
                e = int(p2l[li][s]) if p2l else s
                self._set(li, s, e)
                if e != s:
                    self.fill(li, s, e)
        self.push_tables()
        if torch.cuda.is_available():
            torch.cuda.current_stream(self.device).synchronize()
        self.ready = True
        _log(f"rank {self.rank}: {len(self.layers)} layers x {self.N} slots seeded from "
             f"{placement or 'logical order'} in {time.time() - t0:.1f} s ({self.bytes / 1e9:.2f} GB copied); "
             f"interval {INTERVAL}, at most {MAX_SWAPS} swaps per layer, decay {DECAY}, margin {MARGIN}")
        self.bytes = 0

    # -- policy, between steps ------------------------------------------------------

    def plan_swaps(self, counts: torch.Tensor) -> List[Tuple[int, int, int]]:
        return plan_swaps(np.asarray(counts), self.slot2log, MAX_SWAPS, MARGIN)

    def _collect_counts(self) -> Optional[np.ndarray]:
        """The counts as of the previous round (or None on the first round, or while that copy is
        still in flight); starts this round's copy and decays the device counts."""
        prev = self._round_counts
        if prev is not None and not prev[1].query():
            return None  # the step that carries the copy has not finished: try next round
        out = prev[0].numpy().copy() if prev is not None else None
        buf = prev[0] if prev is not None else torch.empty(self.counts.shape, dtype=torch.float32,
                                                           pin_memory=torch.cuda.is_available())
        buf.copy_(self.counts, non_blocking=True)
        self.counts.mul_(DECAY)
        if self.counts.is_cuda:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
        else:
            ev = _Done()
        self._round_counts = (buf, ev)
        return out

    def before_forward(self, forward_batch) -> None:
        mode = forward_batch.forward_mode
        if not self.ready or not (mode.is_decode() or mode.is_target_verify()):
            return
        self.step += 1
        if self.step % INTERVAL:
            return
        t0 = time.time()
        counts = self._collect_counts()
        if counts is None:
            return
        n = 0
        for li, s, e in plan_swaps(counts, self.slot2log, MAX_SWAPS, MARGIN, layers=self.layers.keys()):
            self._set(li, s, e)
            self.fill(li, s, e)
            n += 1
        if n:
            self.push_tables()
        self.rounds += 1
        self.swaps += n
        self.swap_s += time.time() - t0
        if self.rounds == 1 or (LOG_EVERY and self.rounds % LOG_EVERY == 0) or self.rounds % 64 == 0:
            on_gpu = sum(float(counts[li][[e for e in self.slot2log[li] if e >= 0]].sum()) for li in self.layers)
            _log(f"rank {self.rank}: round {self.rounds} (step {self.step}): {n} swaps, {self.swaps} in all, "
                 f"{self.bytes / 1e9:.2f} GB copied, {self.swap_s * 1e3 / self.rounds:.1f} ms per round; "
                 f"recent routes on the GPU {on_gpu / max(float(counts.sum()), 1.0):.3f}")


class _Done:
    """stands in for the CUDA event of a host-side (CPU tensor) count copy, complete at once"""

    @staticmethod
    def query() -> bool:
        return True


def _physical_order(layer_idx: int, n_experts: int) -> torch.Tensor:
    """Logical expert of each physical slot of the layer (the serving engine's placement map,
    when one is loaded), else the identity."""
    try:
        from sglang.srt.eplb.expert_location_dispatch import get_global_expert_location_metadata
    except ImportError:
        return torch.arange(n_experts)
    meta = get_global_expert_location_metadata()
    if meta is None:
        return torch.arange(n_experts)
    return meta.physical_to_logical_map_cpu[layer_idx].to(torch.int64)


def _reference_lend_mirror(param: torch.Tensor) -> Optional[torch.Tensor]:
    """The host mirror the reference's lend keeps for a device span holding `param`
    (kt_lend.STATE: "dev_spans" device tensors, "bases" their offsets into the "host" bytes),
    as a host view of the parameter's shape, or None when that lend is not loaded or has not
    mirrored yet."""
    try:
        from sglang.srt.layers.moe import kt_lend
    except ImportError:
        return None
    st = getattr(kt_lend, "STATE", None) or {}
    if "host" not in st or "dev_spans" not in st:
        return None
    addr, nbytes = param.data_ptr(), param.numel() * param.element_size()
    for span, base in zip(st["dev_spans"], st["bases"]):
        lo = span.data_ptr()
        if lo <= addr < lo + span.numel():
            off = addr - lo + base
            return st["host"][off:off + nbytes].view(param.dtype).view(param.shape)
    return None


_cache: Optional[HotCache] = None


def register(method, layer) -> Optional[HotCache]:
    """Called by the KT wrapper on its first decode apply of each layer: the cache is built on
    the first call and seeded once every layer has registered. Returns it once ready."""
    global _cache
    if not ENABLED:
        return None
    kt = method.kt_config
    if _cache is None:
        if kt.num_gpu_experts <= 0:
            raise RuntimeError("KT_HOT_DYNAMIC=1 needs GPU expert slots (--kt-num-gpu-experts > 0)")
        _cache = HotCache(kt.num_layers, method.global_num_experts, kt.num_gpu_experts, layer.w13_qweight.device,
                          method.tp_rank)
    if kt.layer_idx not in _cache.layers:
        _cache.layers[kt.layer_idx] = (method.gpu_method, layer)
        if len(_cache.layers) == kt.num_layers:
            _cache.seed(SEED)
    return _cache if _cache.ready else None


def before_forward(forward_batch) -> None:
    if _cache is not None:
        _cache.before_forward(forward_batch)
