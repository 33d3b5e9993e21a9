"""Expert-parallel MoE layer over a process group (one process per GPU, NCCL over NVLink).

Each rank owns a set of expert slots and its own chunk of tokens. A layer call:
  1. routes: owner rank and local slot of every (token, k) route from the placement tables;
     routes to experts no rank owns (ids < 0, or experts left on the CPU) are dropped;
  2. dispatch: each token goes once to every rank that owns at least one of its experts
     (the rank's local expert list and weights travel with it: k slots, -1 padded);
     per-destination counts by one all-to-all, then the rows and the metadata by two more;
  3. local experts: `expert_fn(x_rows, local_ids, local_weights)` -> bf16 rows, the weighted
     sum over the rank's experts of each received token (on the GPU: the tcgen05 prefill
     layer, kt_gguf_moe_multi.moe_prefill, on the rank's slots);
  4. combine: the partial rows go back by the reverse all-to-all and each token's partials
     are summed in fp32 in rank order (deterministic) and rounded once to bf16, together with
     an optional shared expert computed locally.

Placement: `owner[e]` (rank, or -1) and `local[e]` (slot on that rank) for every logical
expert e. `contiguous_placement(E, P)` gives rank g the experts [g*E/P, (g+1)*E/P);
`round_robin_placement(hot, E, P)` spreads a hot list over the ranks; `snake_placement`
deals experts listed hottest first to ranks 0..P-1, P-1..0, ... (config 2 of the benchmark:
the 64 hot experts of a Zipf-skewed router, 8 per rank at 8 ranks).

Two exchanges:
- over peer memory (GPUs, the default with more than one rank): each rank's dispatch kernel
  writes its rows straight into the other ranks' receive buffers, and its combine kernel reads
  its partial outputs straight from their output buffers, over NVLink (kt_ep_dispatch_p2p /
  kt_ep_combine_p2p; the buffers are mapped into every process by CUDA IPC once). The only
  collectives are an all-gather of the per-destination row counts and two one-word
  all-reduces used as barriers (every dispatch before any layer, every layer before any
  combine); the layer reads its row count on the device (kt_moe_prefill_counted), so a call
  makes no host synchronisation. Output buffers alternate between calls, so a rank's next
  layer never overwrites rows another rank is still combining. Capacity: this rank receives
  at most world x (max tokens of any rank) rows, fixed at the first call (max_tokens).
- torch.distributed.all_to_all_single (NCCL, or gloo in the CPU tests; KT_B200_EP_P2P=0 on
  GPUs): counts, rows and metadata by three all-to-alls, the partials back by a fourth; the
  split sizes need one device-to-host copy of the counts per call.
On GPUs the plan, the row packing and the combines are the library's kernels (kt_ep_plan /
kt_ep_pack / kt_ep_combine, csrc/ep.cu); `plan_dispatch` restates the same plan with PyTorch
ops, which the CPU tests of the exchange run on gloo ranks.
"""
import os
from dataclasses import dataclass
from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist


def contiguous_placement(n_experts: int, world: int) -> Tuple[torch.Tensor, torch.Tensor]:
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not split over {world} ranks")
    per = n_experts // world
    e = torch.arange(n_experts, dtype=torch.int32)
    return (e // per).to(torch.int32), (e % per).to(torch.int32)


def round_robin_placement(hot: torch.Tensor, n_experts: int, world: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Hot expert hot[i] goes to rank i % world, slot i // world; the others to no rank."""
    owner = torch.full((n_experts,), -1, dtype=torch.int32)
    local = torch.full((n_experts,), -1, dtype=torch.int32)
    i = torch.arange(hot.numel(), dtype=torch.int32)
    owner[hot.long()] = i % world
    local[hot.long()] = i // world
    return owner, local


def snake_placement(n_experts: int, world: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Experts listed hottest first go to ranks 0..P-1, then P-1..0, and so on (slot = round),
    which balances a skewed load better than plain round-robin."""
    i = torch.arange(n_experts, dtype=torch.int32)
    rnd, pos = i // world, i % world
    owner = torch.where(rnd % 2 == 0, pos, world - 1 - pos).to(torch.int32)
    return owner, rnd.to(torch.int32)


@dataclass
class Dispatch:
    """Host and device bookkeeping of one call (kept for the combine)."""
    send_counts: List[int]
    recv_counts: List[int]
    token_of_row: Optional[torch.Tensor] = None  # CPU path: [n_send] source token of each sent row
    row_of: Optional[torch.Tensor] = None        # GPU path: [T, P] send row of token t for rank r, or -1


def plan_dispatch(topk_ids: torch.Tensor, topk_weights: torch.Tensor, owner: torch.Tensor, local: torch.Tensor,
                  world: int):
    """Rows to send, grouped by destination rank (rank-major, tokens ascending).

    Returns (token_of_row [n], dest_of_row [n], local_ids [n, k] int32, local_w [n, k] fp32,
    send_counts [world] int64 tensor)."""
    T, k = topk_ids.shape
    ids = topk_ids.long()
    valid = ids >= 0
    safe = torch.where(valid, ids, torch.zeros_like(ids))
    dest = torch.where(valid, owner[safe].long(), torch.full_like(ids, -1))  # [T, k]
    lslot = torch.where(valid, local[safe].long(), torch.full_like(ids, -1))
    # sends[r, t]: token t has at least one expert on rank r
    sends = torch.zeros((world, T), dtype=torch.bool, device=topk_ids.device)
    ok = dest >= 0
    rows_t = torch.arange(T, device=topk_ids.device).unsqueeze(1).expand(T, k)
    sends[dest[ok], rows_t[ok]] = True
    dest_of_row, token_of_row = sends.nonzero(as_tuple=True)  # rank-major, tokens ascending
    send_counts = sends.sum(dim=1)
    d = dest[token_of_row]  # [n, k]
    same = d == dest_of_row.unsqueeze(1)
    local_ids = torch.where(same, lslot[token_of_row], torch.full_like(d, -1)).to(torch.int32)
    local_w = torch.where(same, topk_weights[token_of_row].to(torch.float32), torch.zeros_like(d, dtype=torch.float32))
    return token_of_row, dest_of_row, local_ids, local_w, send_counts


class PeerBuffers:
    """The receive and output buffers of one rank's expert-parallel layer, and every rank's
    addresses of them: allocated here, exported with kt_ipc_export, exchanged by one all-gather,
    mapped with kt_ipc_import. peer[b] is a device int64 [world] table of buffer b's address on
    each rank (b: 0 rows, 1 slot ids, 2 weights, 3 and 4 the two alternating outputs)."""

    N_BUF = 5

    def __init__(self, group, world: int, rank: int, rows_cap: int, K: int, k: int, device):
        import ctypes

        from . import _native as N

        self.world, self.rank, self.rows_cap = world, rank, rows_cap
        self.x = torch.empty((rows_cap, K), dtype=torch.bfloat16, device=device)
        self.ids = torch.empty((rows_cap, k), dtype=torch.int32, device=device)
        self.w = torch.empty((rows_cap, k), dtype=torch.float32, device=device)
        self.y = [torch.empty((rows_cap, K), dtype=torch.bfloat16, device=device) for _ in range(2)]
        self.recv_total = torch.zeros(1, dtype=torch.int32, device=device)
        self.counts_all = torch.zeros(world * world, dtype=torch.int32, device=device)
        bufs = [self.x, self.ids, self.w, self.y[0], self.y[1]]
        lib = N.load()
        mine = torch.zeros((self.N_BUF, 9), dtype=torch.int64)  # 64-byte handle, then the offset
        for i, b in enumerate(bufs):
            h = (ctypes.c_uint8 * 64)()
            off = ctypes.c_size_t(0)
            N.check(lib.kt_ipc_export(N.ptr(b), ctypes.cast(h, ctypes.c_void_p), ctypes.byref(off)), "kt_ipc_export")
            mine[i, :8] = torch.frombuffer(bytearray(h), dtype=torch.int64)
            mine[i, 8] = off.value
        every = [torch.empty_like(mine, device=device) for _ in range(world)]
        dist.all_gather(every, mine.to(device), group=group)
        every = [e.cpu() for e in every]
        self._opened = []
        addr = torch.zeros((self.N_BUF, world), dtype=torch.int64)
        for r in range(world):
            for i, b in enumerate(bufs):
                if r == rank:
                    addr[i, r] = b.data_ptr()
                    continue
                h = (ctypes.c_uint8 * 64).from_buffer_copy(every[r][i, :8].numpy().tobytes())
                p = ctypes.c_void_p(0)
                off = int(every[r][i, 8])
                N.check(lib.kt_ipc_import(ctypes.cast(h, ctypes.c_void_p), off, ctypes.byref(p)), "kt_ipc_import")
                self._opened.append((p.value, off))
                addr[i, r] = p.value
        self.peer = addr.to(device)

    def close(self) -> None:
        from . import _native as N

        for p, off in self._opened:
            N.load().kt_ipc_close(p, off)
        self._opened = []


def _p2p_default() -> bool:
    return os.environ.get("KT_B200_EP_P2P", "1") != "0"


class ExpertParallelMoE:
    """One MoE layer, experts sharded over the ranks of `group` (see the module docstring).

    chunks > 1 pipelines the all-to-all exchange: the tokens are split into chunks whose
    all-to-alls run asynchronously (NCCL's stream) while other chunks compute. p2p (default on
    GPUs with more than one rank, KT_B200_EP_P2P=0 turns it off) exchanges over peer memory
    instead; max_tokens bounds the tokens of a call on any rank (default: the largest first
    call)."""

    def __init__(self, owner: torch.Tensor, local: torch.Tensor, expert_fn: Callable, group=None,
                 shared_fn: Optional[Callable] = None, chunks: int = 1, p2p: Optional[bool] = None,
                 max_tokens: Optional[int] = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.owner, self.local = owner, local
        self.expert_fn, self.shared_fn = expert_fn, shared_fn
        self.chunks = max(1, int(chunks))
        self.p2p = _p2p_default() if p2p is None else bool(p2p)
        self.max_tokens = max_tokens
        self.peers: Optional[PeerBuffers] = None
        self.calls = 0
        self._flag = None
        self._dev_tables = None

    # ---- exchange primitives
    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits: List[int], in_splits: List[int], async_op=False):
        if self.world == 1:
            out.copy_(inp)
            return None
        return dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group, async_op=async_op)

    @staticmethod
    def _wait(work):
        if work is not None:
            work.wait()

    # ---- per-chunk steps
    def _plan(self, x, topk_ids, topk_weights):
        """-> dict with counts (device, [P]) and what packing and combining need"""
        dev = x.device
        T, k = topk_ids.shape
        P = self.world
        if x.is_cuda:
            from . import _native as N

            lib = N.load()
            if self._dev_tables is None or self._dev_tables[0].device != dev:
                self._dev_tables = (self.owner.to(dev, torch.int32).contiguous(),
                                    self.local.to(dev, torch.int32).contiguous())
            owner, local = self._dev_tables
            ids = topk_ids.to(torch.int32).contiguous()
            w = topk_weights.to(torch.float32).contiguous()
            ws = N.workspace(lib.kt_ep_plan_workspace_size(T, P), dev)
            counts = torch.empty(P, dtype=torch.int32, device=dev)
            send_token = torch.empty(T * P, dtype=torch.int32, device=dev)
            meta = torch.empty((T * P, 2 * k), dtype=torch.int32, device=dev)
            row_of = torch.empty((T, P), dtype=torch.int32, device=dev)
            N.check(lib.kt_ep_plan(N.ptr(ids), N.ptr(w), T, k, N.ptr(owner), N.ptr(local), owner.numel(), P,
                                   N.ptr(counts), N.ptr(send_token), N.ptr(meta), N.ptr(row_of), N.ptr(ws), ws.numel(),
                                   N.stream_of(x)), "kt_ep_plan")
            return {"counts": counts, "send_token": send_token, "meta": meta, "row_of": row_of, "tok": None}
        owner, local = self.owner.to(dev), self.local.to(dev)
        tok, _, lid, lw, counts = plan_dispatch(topk_ids, topk_weights, owner, local, P)  # the CPU tests
        meta = torch.cat([lid, lw.view(torch.int32)], dim=1).contiguous()
        return {"counts": counts, "send_token": None, "meta": meta, "row_of": None, "tok": tok}

    def _pack(self, x, plan, n_send):
        if x.is_cuda:
            from . import _native as N

            x = x.contiguous()
            out = torch.empty((n_send, x.shape[1]), dtype=x.dtype, device=x.device)
            N.check(N.load().kt_ep_pack(N.ptr(x), x.shape[1], N.ptr(plan["send_token"]), n_send, N.ptr(out),
                                        N.stream_of(x)), "kt_ep_pack")
            return out, plan["meta"][:n_send]
        return x[plan["tok"]].contiguous(), plan["meta"]

    def _combine_rows(self, y_back, plan, send_counts, out, shared):
        """out[t] = bf16(shared[t] + the token's partial rows, fp32 in rank order)"""
        if plan["row_of"] is not None:
            from . import _native as N

            sh = shared.to(out.dtype).contiguous() if shared is not None else None
            N.check(N.load().kt_ep_combine(N.ptr(y_back) if y_back.numel() else None, N.ptr(plan["row_of"]), self.world,
                                           N.ptr(sh), out.shape[0], out.shape[1], N.ptr(out), N.stream_of(out)),
                    "kt_ep_combine")
            return
        acc = torch.zeros(out.shape, dtype=torch.float32, device=out.device)
        if shared is not None:
            acc += shared.float()
        start = 0
        for c in send_counts:  # rank r's rows: each token at most once
            if c:
                idx = plan["tok"][start:start + c]
                acc[idx] += y_back[start:start + c].float()
            start += c
        out.copy_(acc.to(out.dtype))

    # ---- one call, split into phases (for timing) ...
    def dispatch(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor):
        """-> (x_recv [n_recv, K], ids_recv [n_recv, k] int32, w_recv [n_recv, k] fp32, Dispatch)"""
        k = topk_ids.shape[1]
        plan = self._plan(x, topk_ids, topk_weights)
        counts = plan["counts"]
        recv_t = torch.empty_like(counts)
        self._a2a(recv_t, counts, [1] * self.world, [1] * self.world)
        both = torch.stack([counts, recv_t]).cpu()  # the one host sync of the call
        send_counts, recv_counts = both[0].tolist(), both[1].tolist()
        x_send, meta_send = self._pack(x, plan, sum(send_counts))
        x_recv = torch.empty((sum(recv_counts), x.shape[1]), dtype=x.dtype, device=x.device)
        meta_recv = torch.empty((sum(recv_counts), 2 * k), dtype=torch.int32, device=x.device)
        self._a2a(x_recv, x_send, recv_counts, send_counts)
        self._a2a(meta_recv, meta_send, recv_counts, send_counts)
        d = Dispatch(send_counts, recv_counts, plan["tok"], plan["row_of"])
        d.plan = plan
        return x_recv, meta_recv[:, :k].contiguous(), meta_recv[:, k:].contiguous().view(torch.float32), d

    def combine(self, y_recv: torch.Tensor, plan: Dispatch, T: int, shared: Optional[torch.Tensor] = None):
        """partial rows back to their tokens: out[t] = bf16(shared[t] + sum over ranks, in rank order)"""
        y_back = torch.empty((sum(plan.send_counts), y_recv.shape[1]), dtype=y_recv.dtype, device=y_recv.device)
        self._a2a(y_back, y_recv, plan.send_counts, plan.recv_counts)
        out = torch.empty((T, y_recv.shape[1]), dtype=y_recv.dtype, device=y_recv.device)
        self._combine_rows(y_back, plan.plan, plan.send_counts, out, shared)
        return out

    # ---- the exchange over peer memory
    def _barrier(self, dev) -> None:
        """every rank's work so far on its stream before any rank's next step (a one-word
        all-reduce, ordered on the streams like the kernels around it)"""
        if self._flag is None or self._flag.device != dev:
            self._flag = torch.zeros(1, dtype=torch.int32, device=dev)
        dist.all_reduce(self._flag, group=self.group)

    def _peer_buffers(self, T: int, K: int, k: int, dev) -> PeerBuffers:
        if self.peers is None:
            cap = torch.tensor([max(T, self.max_tokens or 0)], dtype=torch.int64, device=dev)
            dist.all_reduce(cap, op=dist.ReduceOp.MAX, group=self.group)
            self.max_tokens = int(cap.item())
            self.peers = PeerBuffers(self.group, self.world, self.rank, self.world * self.max_tokens, K, k, dev)
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the exchange capacity of {self.max_tokens} tokens per rank "
                             f"(max_tokens)")
        return self.peers

    def _call_p2p(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                  events: Optional[list] = None) -> torch.Tensor:
        """events (optional): CUDA events recorded on the stream for phase timing: four (the
        call's start, once the rows are exchanged, after the local layer, the end) or eight (the
        start, after the plan, after the count all-gather, after the dispatch kernel, once the rows
        are exchanged, after the local layer, after the second barrier, the end)."""
        from . import _native as N

        fine = events is not None and len(events) >= 8
        where = {0: 0, 1: 4, 2: 5, 3: 7} if fine else {0: 0, 1: 1, 2: 2, 3: 3}

        def mark(i):
            if events is not None:
                events[where[i]].record()

        def mark_fine(i):
            if fine:
                events[i].record()

        T, K = x.shape
        k = topk_ids.shape[1]
        dev = x.device
        pb = self._peer_buffers(T, K, k, dev)
        lib = N.load()
        st = N.stream_of(x)
        x = x.contiguous()
        mark(0)
        plan = self._plan(x, topk_ids, topk_weights)
        mark_fine(1)
        dist.all_gather_into_tensor(pb.counts_all, plan["counts"], group=self.group)
        mark_fine(2)
        N.check(lib.kt_ep_dispatch_p2p(N.ptr(x), K, N.ptr(plan["send_token"]), N.ptr(plan["meta"]), k,
                                       N.ptr(pb.counts_all), self.rank, self.world, N.ptr(pb.peer[0]),
                                       N.ptr(pb.peer[1]), N.ptr(pb.peer[2]), pb.rows_cap, N.ptr(pb.recv_total), st),
                "kt_ep_dispatch_p2p")
        mark_fine(3)
        self._barrier(dev)  # every rank's rows are in place
        mark(1)
        b = self.calls % 2
        self.expert_fn.counted(pb.x, pb.recv_total, pb.ids, pb.w, pb.y[b])
        shared = self.shared_fn(x) if self.shared_fn is not None else None
        mark(2)
        self._barrier(dev)  # every rank's partial outputs are in place
        mark_fine(6)
        out = torch.empty((T, K), dtype=x.dtype, device=dev)
        sh = shared.to(x.dtype).contiguous() if shared is not None else None
        N.check(lib.kt_ep_combine_p2p(N.ptr(plan["row_of"]), N.ptr(pb.counts_all), self.rank, self.world,
                                      N.ptr(pb.peer[3 + b]), N.ptr(sh), T, K, N.ptr(out), st), "kt_ep_combine_p2p")
        mark(3)
        self.calls += 1
        return out

    def close(self) -> None:
        """Unmaps the other ranks' buffers (after the last call, on every rank)."""
        if self.peers is not None:
            torch.cuda.synchronize()
            self.peers.close()
            self.peers = None

    # ---- ... or pipelined over chunks
    def __call__(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor) -> torch.Tensor:
        T, K = x.shape
        k = topk_ids.shape[1]
        if self.world > 1 and x.is_cuda and self.p2p and self.chunks == 1:
            return self._call_p2p(x, topk_ids, topk_weights)
        if self.world == 1 and x.is_cuda and self.shared_fn is None:
            # one rank: no exchange; the local slots straight from the logical ids
            # ids outside [0, n_experts) are dropped, as kt_ep_plan drops them on the multi-rank path
            local = self.local.to(x.device, torch.int32)
            owned = self.owner.to(x.device) == 0
            n = owned.numel()
            ids = topk_ids.long()
            safe = ids.clamp(0, n - 1)
            valid = (ids >= 0) & (ids < n) & owned[safe]
            lid = torch.where(valid, local[safe], torch.full_like(topk_ids, -1, dtype=torch.int32))
            return self.expert_fn(x.contiguous(), lid.to(torch.int32).contiguous(),
                                  topk_weights.to(torch.float32).contiguous())
        C = min(self.chunks, max(1, T))
        bounds = [(T * c // C, T * (c + 1) // C) for c in range(C)]
        # 1. plans and counts of every chunk, one host sync for all
        plans, recvs, works = [], [], []
        for a, b in bounds:
            p = self._plan(x[a:b], topk_ids[a:b], topk_weights[a:b])
            r = torch.empty_like(p["counts"])
            works.append(self._a2a(r, p["counts"], [1] * self.world, [1] * self.world, async_op=True))
            plans.append(p)
            recvs.append(r)
        for w in works:
            self._wait(w)
        allc = torch.stack([torch.cat([p["counts"], r]) for p, r in zip(plans, recvs)]).cpu()
        sends = [row[:self.world].tolist() for row in allc]
        recvc = [row[self.world:].tolist() for row in allc]
        # 2. pack and dispatch every chunk (asynchronous all-to-alls)
        rx, rmeta, wd = [], [], []
        for c, (a, b) in enumerate(bounds):
            xs, ms = self._pack(x[a:b], plans[c], sum(sends[c]))
            xr = torch.empty((sum(recvc[c]), K), dtype=x.dtype, device=x.device)
            mr = torch.empty((sum(recvc[c]), 2 * k), dtype=torch.int32, device=x.device)
            wd.append((self._a2a(xr, xs, recvc[c], sends[c], async_op=True),
                       self._a2a(mr, ms, recvc[c], sends[c], async_op=True), xs, ms))
            rx.append(xr)
            rmeta.append(mr)
        # 3. experts of chunk c once its rows are here; its partials go back asynchronously
        backs, wb = [], []
        for c in range(C):
            self._wait(wd[c][0])
            self._wait(wd[c][1])
            if rx[c].shape[0]:
                y = self.expert_fn(rx[c], rmeta[c][:, :k].contiguous(), rmeta[c][:, k:].contiguous().view(torch.float32))
            else:
                y = torch.empty((0, K), dtype=x.dtype, device=x.device)
            yb = torch.empty((sum(sends[c]), K), dtype=x.dtype, device=x.device)
            wb.append((self._a2a(yb, y, sends[c], recvc[c], async_op=True), y))
            backs.append(yb)
        shared = self.shared_fn(x) if self.shared_fn is not None else None
        # 4. combine
        out = torch.empty((T, K), dtype=x.dtype, device=x.device)
        for c, (a, b) in enumerate(bounds):
            self._wait(wb[c][0])
            self._combine_rows(backs[c], plans[c], sends[c], out[a:b], shared[a:b] if shared is not None else None)
        return out


def prefill_expert_fn(w13: torch.Tensor, w2: torch.Tensor, type13: int, type2: int, inter: int):
    """The rank's slots through the tcgen05 prefill layer (bf16 rows)."""
    from . import kt_gguf_moe_multi as M
    from . import _native as N

    cache = {}

    def workspace(T, k, dev):
        need = N.load().kt_moe_prefill_workspace_size(T, k, w2.shape[1], inter, w13.shape[0])
        ws = cache.get("ws")
        if ws is None or ws.numel() < need:
            ws = cache["ws"] = N.workspace(max(need, int(need * 1.25)), dev)
        return ws

    def fn(x, ids, w):
        T, k = ids.shape
        return M.moe_prefill(x, w13, w2, ids, w, type13, type2, inter, workspace=workspace(T, k, x.device))

    def counted(x, n_dev, ids, w, out):
        """the layer over the first n_dev[0] rows of x / ids / w (a device count), into out"""
        cap, k = ids.shape
        ws = workspace(cap, k, x.device)
        N.check(N.load().kt_moe_prefill_counted(N.ptr(x), cap, N.ptr(n_dev), x.shape[1], inter, N.ptr(ids), N.ptr(w), k,
                                                N.ptr(w13), type13, N.ptr(w2), type2, 0, w13.shape[0], N.ptr(out),
                                                N.ptr(ws), ws.numel(), N.stream_of(x)), "kt_moe_prefill_counted")
        return out

    fn.counted = counted
    return fn
