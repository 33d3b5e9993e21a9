"""Per-layer weight return for prefill: layer weights that live in pinned host memory are copied
into one of two device slots on a side stream while the previous layer computes.

The lend pipeline of the reference (kt_lend.py `_prefetch` / `_enter`, lines 1298-1350) keeps
each layer's bf16 weights in a pinned host buffer during prefill and brings them back one
layer ahead: slot i % 2 holds layer i; the copy of layer i+1 starts when layer i starts and
waits for the compute stream to be done with layer i-1 (the slot's previous occupant); the
compute stream waits for the copy of layer i before layer i runs. `LayerStreamer` is that
protocol with CUDA events:

    s = LayerStreamer(host_weights, device)     # host_weights[i]: pinned tensor of layer i
    for i in range(n_layers):
        w = s.enter(i)                           # device copy of layer i (slot i % 2)
        ...layer i on the current stream...
    s.finish()

The copies are plain cudaMemcpyAsync (torch copy_ from pinned memory, non_blocking) on the
side stream, one per layer, so they overlap the compute stream's kernels. With timing=True,
`stats()` reports the bytes copied, the time the copies took on the side stream and the time
the compute stream spent waiting for them (the part of the copy time not hidden).
"""
from typing import Dict, List, Optional, Tuple

import torch


class LayerStreamer:
    def __init__(self, host_weights: List[torch.Tensor], device: torch.device, timing: bool = False):
        if not host_weights:
            raise ValueError("no layers")
        shape, dtype = host_weights[0].shape, host_weights[0].dtype
        for h in host_weights:
            if h.shape != shape or h.dtype != dtype:
                raise ValueError("all layers must have one shape and dtype (one slot size)")
            if not h.is_pinned():
                raise ValueError("host weights must be in pinned memory (asynchronous copies)")
        self.host = host_weights
        self.device = device
        self.timing = timing
        self.slots = [torch.empty(shape, dtype=dtype, device=device) for _ in range(2)]
        self.side = torch.cuda.Stream(device=device)
        self.done: List[Optional[torch.cuda.Event]] = [None, None]  # compute stream done with slot k
        self.copy_end: Dict[int, torch.cuda.Event] = {}
        self.cur: Optional[int] = None
        self.copies: List[Tuple[torch.cuda.Event, torch.cuda.Event, int]] = []  # (start, end, bytes)
        self.waits: List[Tuple[torch.cuda.Event, torch.cuda.Event]] = []

    def _prefetch(self, i: int) -> None:
        if i >= len(self.host) or i in self.copy_end:
            return
        k = i % 2
        with torch.cuda.stream(self.side):
            if self.done[k] is not None:
                self.side.wait_event(self.done[k])
            start = torch.cuda.Event(enable_timing=self.timing)
            start.record(self.side)
            self.slots[k].copy_(self.host[i], non_blocking=True)
            end = torch.cuda.Event(enable_timing=self.timing)
            end.record(self.side)
        self.copy_end[i] = end
        self.copies.append((start, end, self.host[i].numel() * self.host[i].element_size()))

    def enter(self, i: int) -> torch.Tensor:
        """Layer i is about to run on the current stream: returns its device weights."""
        cur = torch.cuda.current_stream(self.device)
        if self.cur is not None:
            ev = torch.cuda.Event()
            ev.record(cur)
            self.done[self.cur % 2] = ev  # the previous layer's slot is free after this point
        if self.cur is None or i <= self.cur:
            self.copy_end = {}  # a new pass over the layers
        if i not in self.copy_end:
            self.side.wait_stream(cur)  # nothing prefetched: order after the compute stream's past
            self._prefetch(i)
        if self.timing:
            before = torch.cuda.Event(enable_timing=True)
            before.record(cur)
        cur.wait_event(self.copy_end[i])
        if self.timing:
            after = torch.cuda.Event(enable_timing=True)
            after.record(cur)
            self.waits.append((before, after))
        self.cur = i
        self._prefetch(i + 1)
        return self.slots[i % 2]

    def finish(self) -> None:
        """The pass is over: the last layer's slot is released to the next pass."""
        if self.cur is not None:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self.done[self.cur % 2] = ev
        self.cur = None
        self.copy_end = {}

    def stats(self) -> dict:
        """After a synchronize: bytes copied, copy time on the side stream, compute-stream wait."""
        if not self.timing:
            raise RuntimeError("LayerStreamer(timing=True) records the events")
        copy_ms = sum(s.elapsed_time(e) for s, e, _ in self.copies)
        wait_ms = sum(b.elapsed_time(a) for b, a in self.waits)
        nbytes = sum(n for _, _, n in self.copies)
        return {"bytes": nbytes, "copies": len(self.copies), "copy_ms": copy_ms, "wait_ms": wait_ms,
                "h2d_GBps": nbytes / (copy_ms * 1e-3) / 1e9 if copy_ms > 0 else None,
                "hidden_frac": 1.0 - wait_ms / copy_ms if copy_ms > 0 else None}
