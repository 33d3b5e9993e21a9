"""Streamed prefill of the GGUF experts that are not resident on the GPU — B200 implementation.

Drop-in for sglang.srt.layers.moe.kt_stream_prefill_gguf (the reference's SGLang tree,
flash-next-gguf patch, KTStreamPrefillGGUF and stream_prefill_for / stream_prefill_init_early):
a prefill chunk of at least KT_GPU_STREAM_PREFILL tokens runs every non-resident expert of
the layer on the GPU by streaming its raw GGUF bytes from pinned host banks, group by group.

The reference stages a group's raw bytes, dequantizes them to bf16 weights in HBM (Triton)
and runs FlashInfer's CUTLASS fused MoE, adding each group's bf16 output into a bf16
accumulator. Here a group is one kt_moe_prefill_ex call on the staged raw bytes: the tcgen05
GEMMs dequantize in shared memory, so nothing but the raw bytes crosses PCIe or HBM, and the
sum over groups is carried in fp32 and rounded to bf16 once.

Layout:
  bank (per layer, pinned, physical expert order): w13 [E, 2N * row_bytes(K)] with each
    expert's gate rows then up rows (the slot layout of w13_qweight, so a group is ONE copy),
    w2 [E, K * row_bytes(N)];
  two device slots of GROUP experts each; group g is copied into slot g % 2 on a copy stream
  while group g - 1 computes on the caller's stream, ordered by CUDA events (the copy into a
  slot waits for the compute that last read it; the compute waits for its copy).

Env (names of the reference): KT_GPU_STREAM_PREFILL (threshold in tokens; 0 = off),
KT_GPU_STREAM_GROUP (experts per group; default 32 here, 8 in the reference: on a B200 with
config 2's 192 streamed experts, groups of 8 / 16 / 32 reached 0.89 / 0.96 / 0.99 of a plain
pinned copy of the same bytes, the smaller groups losing to per-group copy and launch gaps;
two slots of 32 such experts are 128 MB), KT_GPU_STREAM_TIMING,
KT_GPU_STREAM_EARLY_INIT, and KT_GPU_STREAM_SELFTEST=2: the first streamed layer of the process
is recomputed by an independent path (each used expert's bank bytes dequantized on the GPU
by kt_gguf_dequantize, then plain fp32 matmuls, SwiGLU and the weighted sum in torch) and the
rel-L2 and cosine of the streamed output against it are logged and kept in `last_check` (the
reference's _reference_check, its in-serving numerical guard on this path). The reference's per-group CUDA graphs (and the row padding,
KT_GPU_STREAM_ROW_STEP, that keeps their count small) are not needed: a group is four
kernel launches through the C ABI.
"""
import os
import time
import traceback
from typing import Dict, List, Optional

import torch

from . import _native as N
from . import kt_gguf_moe_multi as _multi

STREAM_THRESHOLD = int(os.environ.get("KT_GPU_STREAM_PREFILL", "0") or 0)
GROUP_SIZE = int(os.environ.get("KT_GPU_STREAM_GROUP", "32") or 32)
TIMING = os.environ.get("KT_GPU_STREAM_TIMING") == "1"
EARLY_INIT = os.environ.get("KT_GPU_STREAM_EARLY_INIT", "0") == "1"
SELFTEST = os.environ.get("KT_GPU_STREAM_SELFTEST", "0")


def _log(msg: str):
    print(f"[kt-stream-gguf {time.strftime('%H:%M:%S')}] {msg}", flush=True)


def _align64(n: int) -> int:
    return (n + 63) & ~63


class _Slot:
    """Device bytes for GROUP experts: w13 and w2 regions, and the two events that order it."""

    def __init__(self, G: int, strides, device):
        self.raw = [torch.empty((G * st,), dtype=torch.uint8, device=device) for st in strides]
        self.dma_done = torch.cuda.Event()
        self.compute_done = torch.cuda.Event()
        self.compute_used = False


class KTStreamPrefillGGUF:
    """Per-rank streaming state, shared by every MoE layer (hot/kt_gguf_hot.py's method supplies
    the GGUF reader, this rank's N / K slice and the layer types)."""

    def __init__(self, method, layer=None, group_size: Optional[int] = None):
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.reader = method.reader
        self.rank = method.rank
        self.world = method.world
        self.N, self.K = method.N, method.K
        self.E = self.reader.E
        self.G = int(group_size or GROUP_SIZE)
        if self.G <= 0:
            raise ValueError("the group size must be positive")
        self._layer_types: Dict[int, tuple] = {}
        self._part_bytes: Dict[int, tuple] = {}
        self._banks: Dict[int, List[torch.Tensor]] = {}
        self._strides = [0, 0]
        self.slots: List[_Slot] = []
        self.transfer_stream = torch.cuda.Stream(device=self.device)
        self._acc: Dict[int, torch.Tensor] = {}
        self._workspace = None
        self.calls = 0
        self.bytes_staged = 0
        self.last_check: Optional[dict] = None  # the self-check's result (KT_GPU_STREAM_SELFTEST=2)

    # -- geometry -----------------------------------------------------------

    def _geometry(self, layer_idx: int):
        types = self._layer_types.get(layer_idx)
        if types is None:
            t = tuple(int(v) for v in self.reader.types(layer_idx))
            if t[0] != t[1]:
                raise RuntimeError(f"layer {layer_idx}: gate {t[0]} and up {t[1]} differ")
            for v in (t[0], t[2]):
                if v not in N.PREFILL_TYPES:
                    raise RuntimeError(f"layer {layer_idx}: ggml type {v} has no B200 prefill kernel "
                                       f"(supported: {sorted(N.PREFILL_TYPES)})")
            pb = (2 * self.N * N.row_bytes(t[0], self.K), self.K * N.row_bytes(t[2], self.N))
            self._layer_types[layer_idx], self._part_bytes[layer_idx] = (t[0], t[2]), pb
            grow = [max(self._strides[i], _align64(pb[i])) for i in range(2)]
            if grow != self._strides:  # slots sized for the largest layer seen
                if self.slots:  # copies or groups may still read the old slots
                    torch.cuda.synchronize(self.device)
                self._strides = grow
                self.slots = [_Slot(self.G, self._strides, self.device) for _ in range(2)]
            types = self._layer_types[layer_idx]
        return types, self._part_bytes[layer_idx]

    def _physical_to_logical(self, layer_idx: int) -> Optional[torch.Tensor]:
        try:
            from sglang.srt.eplb.expert_location_dispatch import get_global_expert_location_metadata
        except ImportError:
            return None
        meta = get_global_expert_location_metadata()
        if meta is None:
            return None
        m = meta.physical_to_logical_map_cpu[layer_idx].to(torch.int64)
        return None if torch.equal(m, torch.arange(m.numel(), dtype=torch.int64)) else m

    # -- banks --------------------------------------------------------------

    def _bank(self, layer_idx: int) -> List[torch.Tensor]:
        """This rank's slice of every expert of the layer, pinned, physical order:
        [w13 [E, 2N*row_bytes(K)] (gate rows then up rows per expert), w2 [E, K*row_bytes(N)]]."""
        b = self._banks.get(layer_idx)
        if b is not None:
            return b
        t0 = time.time()
        _, pb = self._geometry(layer_idx)
        p2l = self._physical_to_logical(layer_idx)
        experts = p2l if p2l is not None else torch.arange(self.E)
        pin = torch.cuda.is_available()
        w13 = torch.empty((self.E, pb[0]), dtype=torch.uint8, pin_memory=pin)
        half = pb[0] // 2
        w13[:, :half].copy_(self.reader.slice(layer_idx, "gate", self.N, self.rank, experts).reshape(self.E, -1))
        w13[:, half:].copy_(self.reader.slice(layer_idx, "up", self.N, self.rank, experts).reshape(self.E, -1))
        w2 = torch.empty((self.E, pb[1]), dtype=torch.uint8, pin_memory=pin)
        w2.copy_(self.reader.slice(layer_idx, "down", self.N, self.rank, experts).reshape(self.E, -1))
        b = self._banks[layer_idx] = [w13, w2]
        if TIMING:
            _log(f"rank {self.rank}: layer {layer_idx} bank {(pb[0] + pb[1]) * self.E / 1e9:.2f} GB pinned in "
                 f"{time.time() - t0:.1f} s")
        return b

    def build_all_banks(self, layers) -> None:
        """Every listed layer's bank (the reference builds them at load with threads; the copies
        out of the GGUF mapping release the GIL)."""
        from concurrent.futures import ThreadPoolExecutor

        layers = list(layers)
        for li in layers:
            self._geometry(li)
        with ThreadPoolExecutor(max_workers=max(1, min(8, len(layers)))) as ex:
            list(ex.map(self._bank, layers))

    # -- staging ------------------------------------------------------------

    def _stage(self, layer_idx: int, gi: int, base: int, n: int, stats) -> None:
        """Group gi's raw bytes (experts [base, base + n)) into slot gi % 2 on the copy stream."""
        banks = self._bank(layer_idx)
        _, pb = self._geometry(layer_idx)
        slot = self.slots[gi % 2]
        t0 = time.perf_counter()
        with torch.cuda.stream(self.transfer_stream):
            if slot.compute_used:
                self.transfer_stream.wait_event(slot.compute_done)
            for i in range(2):
                slot.raw[i][:n * pb[i]].view(n, pb[i]).copy_(banks[i][base:base + n], non_blocking=True)
            slot.dma_done.record(self.transfer_stream)
        self.bytes_staged += n * (pb[0] + pb[1])
        stats["dma_enq"] += time.perf_counter() - t0

    # -- one group ----------------------------------------------------------

    def _group_body(self, layer_idx: int, gi: int, base: int, n: int, g: dict, acc_flags: int) -> None:
        slot = self.slots[gi % 2]
        (type13, type2), pb = self._geometry(layer_idx)
        w13 = slot.raw[0][:n * pb[0]].view(n, 2 * self.N, -1)
        w2 = slot.raw[1][:n * pb[1]].view(n, self.K, -1)
        _multi.moe_prefill_ex(g["x"], w13, w2, g["ids"], g["w"], type13, type2, self.N, id_base=base, acc=g["acc"],
                              acc_flags=acc_flags, out=g["out"], workspace=self._ws(g["x"].shape[0], g["ids"].shape[1]))

    def _ws(self, T: int, top_k: int) -> torch.Tensor:
        need = N.load().kt_moe_prefill_workspace_size(T, top_k, self.K, self.N, self.G)
        if self._workspace is None or self._workspace.numel() < need:
            self._workspace = N.workspace(need, self.device)
        return self._workspace

    # -- one layer ----------------------------------------------------------

    def groups(self, first: int):
        return [(b, min(self.G, self.E - b)) for b in range(first, self.E, self.G)]

    def run(self, method, layer, dispatch_output, physical_ids: torch.Tensor) -> torch.Tensor:
        """Sum of the streamed experts' outputs for this layer, bf16 [tokens, hidden]. Streams the
        experts from num_gpu_experts on (from 0 when the method streams its hot experts too);
        physical_ids [T, k] are the router's ids in physical order (every expert, none masked)."""
        x = dispatch_output.hidden_states
        if x.dtype != torch.bfloat16:
            raise TypeError("the streamed prefill takes bf16 activations")
        T = x.shape[0]
        layer_idx = method.kt_config.layer_idx
        topk_weights = dispatch_output.topk_output.topk_weights
        first = 0 if getattr(method, "streams_hot_experts", False) else method.num_gpu_experts
        groups = self.groups(first)
        out = torch.empty((T, self.K), dtype=torch.bfloat16, device=x.device)
        if not groups:
            return out.zero_()
        stats = {"dma_enq": 0.0, "enq": 0.0}
        t0 = time.perf_counter()
        self._bank(layer_idx)
        acc = self._acc.get(T)
        if acc is None:
            acc = self._acc[T] = torch.empty((T, self.K), dtype=torch.float32, device=x.device)
        g = {"x": x.contiguous(), "ids": physical_ids.to(torch.int32).contiguous(),
             "w": topk_weights.to(torch.float32).contiguous(), "acc": acc, "out": out}
        cur = torch.cuda.current_stream(self.device)
        self._stage(layer_idx, 0, groups[0][0], groups[0][1], stats)
        last = len(groups) - 1
        for gi, (base, n) in enumerate(groups):
            slot = self.slots[gi % 2]
            t1 = time.perf_counter()
            cur.wait_event(slot.dma_done)
            if last == 0:
                flags = 0
            elif gi == 0:
                flags = N.KT_ACC_STORE
            elif gi < last:
                flags = N.KT_ACC_LOAD | N.KT_ACC_STORE
            else:
                flags = N.KT_ACC_LOAD
            self._group_body(layer_idx, gi, base, n, g, flags)
            slot.compute_done.record(cur)
            slot.compute_used = True
            stats["enq"] += time.perf_counter() - t1
            if gi + 1 < len(groups):
                self._stage(layer_idx, gi + 1, groups[gi + 1][0], groups[gi + 1][1], stats)
        self.calls += 1
        if SELFTEST == "2" and self.last_check is None:
            self._self_check(layer_idx, first, g, out)
        if TIMING:
            cur.synchronize()
            _log(f"rank {self.rank} layer {layer_idx} tokens={T} groups={len(groups)} dma_enq={stats['dma_enq'] * 1e3:.1f}ms "
                 f"enq={stats['enq'] * 1e3:.1f}ms total={(time.perf_counter() - t0) * 1e3:.1f}ms")
        return out


    # -- self-check ---------------------------------------------------------

    def _self_check(self, layer_idx: int, first: int, g: dict, out: torch.Tensor) -> dict:
        """The streamed experts' output of this call recomputed from the bank bytes by an
        independent path: each used expert dequantized on the GPU to fp32 (kt_gguf_dequantize,
        bit-exact to ggml), then fp32 matmuls, SwiGLU and the fp32 weighted sum in torch."""
        from . import kernels as Kn

        torch.cuda.current_stream(self.device).synchronize()
        (type13, type2), _ = self._geometry(layer_idx)
        banks = self._bank(layer_idx)
        x, ids, w = g["x"].float(), g["ids"].long(), g["w"]
        ref = torch.zeros((x.shape[0], self.K), dtype=torch.float32, device=x.device)
        used = 0
        for e in range(first, self.E):
            tok, kk = torch.where(ids == e)
            if tok.numel() == 0:
                continue
            used += 1
            w13 = Kn.gguf_dequantize(banks[0][e].to(x.device).view(2 * self.N, -1), type13, self.K, torch.float32)
            w2 = Kn.gguf_dequantize(banks[1][e].to(x.device).view(self.K, -1), type2, self.N, torch.float32)
            xe = x[tok]
            h = torch.nn.functional.silu(xe @ w13[:self.N].t()) * (xe @ w13[self.N:].t())
            ref.index_add_(0, tok, (h @ w2.t()) * w[tok, kk].unsqueeze(1))
        got = out.float()
        rel = float((got - ref).norm() / ref.norm().clamp_min(1e-30))
        cos = float(torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0))
        self.last_check = {"layer": layer_idx, "tokens": int(x.shape[0]), "experts_used": used, "rel_l2": rel,
                           "cosine": cos}
        _log(f"rank {self.rank}: self-check layer {layer_idx}, {x.shape[0]} tokens, {used} streamed experts: "
             f"rel-L2 {rel:.2e}, cosine {cos:.6f} against fp32 dequant + matmul")
        return self.last_check


_instance: Optional[KTStreamPrefillGGUF] = None
_failed = False


def stream_prefill_init_early(method, layer) -> None:
    """KT_GPU_STREAM_EARLY_INIT=1: build the streamer and every layer's bank at load time."""
    global _instance, _failed
    if not EARLY_INIT or STREAM_THRESHOLD <= 0 or _failed or _instance is not None:
        return
    t0 = time.time()
    try:
        _instance = KTStreamPrefillGGUF(method, layer)
        _instance.build_all_banks(getattr(method.reader, "layers", [method.kt_config.layer_idx]))
    except Exception:
        _failed = True
        _log("early init failed:\n" + traceback.format_exc())
        raise
    _log(f"rank {_instance.rank}: GGUF streamer built at load time in {time.time() - t0:.0f} s")


def stream_prefill_for(method, layer, num_tokens: int) -> Optional[KTStreamPrefillGGUF]:
    """The process's streamer when this call qualifies (num_tokens >= KT_GPU_STREAM_PREFILL, not
    inside a CUDA graph capture), else None."""
    global _instance, _failed
    if STREAM_THRESHOLD <= 0 or _failed:
        return None
    if num_tokens < STREAM_THRESHOLD or torch.cuda.is_current_stream_capturing():
        return None
    if _instance is None:
        try:
            _instance = KTStreamPrefillGGUF(method, layer)
        except Exception:
            _failed = True
            _log("init failed:\n" + traceback.format_exc())
            raise
    return _instance
