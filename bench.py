#!/usr/bin/env python
"""MoE-layer prefill throughput (tokens/s) at a 16K-token chunk — BASELINE config 2.

Workload: one Qwen3.5-35B-A3B-like MoE layer: hidden 2048, expert intermediate 512, 256
experts top-8 (softmax), 64 experts resident on the GPU (the rest masked to -1 as for CPU
experts), gate/up Q4_K and down Q6_K GGUF blocks, router logits N(0,1) plus a log-space
Zipf(1.1) per-expert bias, bf16 activations N(0,1), weights N(0,0.02) quantized with the
package's encoders. All data synthetic and seeded (no checkpoint is available here).

A step = one kt_moe_prefill call over the chunk (routing permutation, tcgen05 gate/up
GEMM with SwiGLU, tcgen05 down GEMM, combine), inputs resident in HBM. With --gpus N > 1 the
layer runs expert-parallel (kt_gguf_b200.ep): the 64 resident experts are dealt over the ranks
hottest first in snake order, each rank routes its own 16K-token chunk, and tokens and partial
outputs travel by NCCL all-to-all ("scaling": "weak": per-rank tokens fixed as ranks are
added); the time is the max over ranks of CUDA-event time. --replicas runs N independent
token-parallel replicas instead (no data-path collective), and --config 4 the
DeepSeek-V3-like layer expert-parallel.

Parity at the headline size: after the timed run, 256 tokens spread evenly over the chunk
are recomputed on the CPU by the fp32 dequant-then-matmul oracle and by the restated
reference arithmetic (q8_1 GEMVs, bf16 intermediates), and the line reports the rel-L2 of
the GPU layer against both and of the reference arithmetic against fp32.

--config 1 / 3 print the other BASELINE configurations (one JSON line per point): config 1
(Q8_0, 256 tokens, with the CPU baseline on the whole chunk and the rel-L2 against the fp32
oracle) and config 3 (IQ3_S, 512 experts top-10: the decode GEMV at M = 1, 4, 16, 64 against
the HBM roofline with L2 flushed before every call, and the prefill GEMMs at M = 2048, 16384).

--impl reference times the reference's CPU implementation of the path as restated in
oracle/ (the reference's own CPU expert library, kt-kernel + llama.cpp, ships only as
patches on un-vendored sources and cannot be built here) on the host cores: the q8_1 x GGUF
integer-dot arithmetic with AVX-512 VNNI dot products (oracle/kt_cpu_simd.c) where the host
has them, else the scalar restatement. The same implementation is the cpu_baseline of the
headline line.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "kt-prefill-lend_b200"))

METRIC = "MoE-layer prefill tok/s @16K chunk"
# name of the first stage by kt_moe_prefill_predequant's bits: the permutation, then the weight
# passes
PASS_STAGE = {1: "permute_and_w13_bf16_pass", 3: "permute_and_bf16_weight_passes"}
CONFIG_NAME = "qwen3.5-35b-a3b-like MoE layer (BASELINE configs[1])"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample", type=int, default=256, help="tokens per CPU-baseline sample")
    ap.add_argument("--tokens", type=int, default=16384, help="chunk size (profiling runs use smaller chunks)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end pass (profiling)")
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5],
                    help="2: the headline line (default); 1 and 3: the other BASELINE configs, one JSON line per point")
    ap.add_argument("--m-list", default="1,4,16,64,2048,16384",
                    help="sweep token counts (config 3, or config 2 with --sweep): below 128 the decode GEMV, "
                         "from 128 the prefill GEMMs")
    ap.add_argument("--tokens-c4", type=int, default=32768, help="config 4: tokens per rank")
    ap.add_argument("--ep", action="store_true", help="config 2 expert-parallel (NCCL all-to-all) even at one GPU "
                                                      "(the default from two GPUs)")
    ap.add_argument("--replicas", action="store_true", help="N > 1: token-parallel replicas of the whole layer "
                                                            "instead of the expert-parallel split")
    ap.add_argument("--ep-chunks", type=int, default=1, help="expert-parallel runs: token chunks per call whose "
                                                             "all-to-alls overlap the other chunks' GEMMs")
    ap.add_argument("--sweep", action="store_true", help="config 2: run the decode/prefill sweep instead of the "
                                                         "headline line")
    ap.add_argument("--stream", action="store_true", help="config 2 with the 192 non-resident experts streamed "
                                                          "from pinned host banks (kt_stream_prefill_gguf)")
    ap.add_argument("--group", type=int, default=0, help="--stream: experts per group (0: KT_GPU_STREAM_GROUP)")
    return ap.parse_args()


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def profile_traffic(name: str):
    """per-launch DRAM bytes of a kernel from the committed ncu summary, or None"""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch_full_size:"):
            return float(line.split(":", 1)[1].strip())
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons for one GPU, sampled every 50 ms by one
    streaming nvidia-smi process during the timed region"""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.samples = []
        self._proc = None
        self._t = None

    def _run(self):
        for line in self._proc.stdout:
            f = [x.strip() for x in line.strip().split(",")]
            if len(f) == 7:
                try:
                    self.samples.append((time.time(), float(f[0]), float(f[1]), f[3:]))
                except ValueError:
                    pass

    def start(self):
        try:
            self._proc = subprocess.Popen(["nvidia-smi", "-i", self.uuid, f"--query-gpu={self.FIELDS}",
                                           "--format=csv,noheader,nounits", "-lms", "50"],
                                          stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            return
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()

    def stop(self, t0, t1):
        if self._proc:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._t:
            self._t.join(timeout=5)
        win = [s for s in self.samples if t0 <= s[0] <= t1] or self.samples
        if not win:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for s in win for n, v in zip(names, s[3]) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(s[1] for s in win), "sm_max_mhz": max(s[2] for s in win),
                "reasons": reasons, "samples": len(win)}


def spread_tokens(T: int, n: int):
    """n token indices spread evenly over a chunk of T tokens"""
    import numpy as np

    return np.unique(np.linspace(0, T - 1, min(n, T)).round().astype(np.int64))


def cpu_layer_fn():
    """the timed CPU implementation of the layer: the reference's arithmetic with AVX-512 VNNI
    dot products (oracle/kt_cpu_simd.c) where the host has them, else the scalar restatement;
    -> (function, kind label)"""
    from oracle import oracle as O

    O.build()
    if O.simd_available():
        return O.moe_cpu_simd, ("AVX-512 VNNI restatement of the reference's CPU arithmetic class (kt-kernel's "
                                "q8_1 x GGUF integer dots), OpenMP over the host cores")
    return O.moe_ref_bf16, "scalar restatement of the reference's q8_1 x GGUF integer-dot arithmetic, OpenMP"


def cpu_baseline(L, idx, threads):
    """the CPU implementation of the layer on the tokens idx -> (tokens/s, description)"""
    import numpy as np
    import torch

    os.environ["OMP_NUM_THREADS"] = str(threads)
    fn, kind = cpu_layer_fn()
    xb = L.x[idx].view(torch.int16).numpy().view(np.uint16)
    ids = L.topk_ids[idx].numpy()
    w = L.topk_weights[idx].numpy()
    fn(xb[:8], ids[:8], w[:8], L.type13, L.w13, L.type2, L.w2, L.inter)  # warm-up
    times = []
    for _ in range(3):
        t = time.perf_counter()
        fn(xb, ids, w, L.type13, L.w13, L.type2, L.w2, L.inter)
        times.append(time.perf_counter() - t)
    return len(idx) / min(times), kind


def headline_parity(L, idx, out_rows, ref_bits):
    """rel-L2 of the GPU layer's rows (bf16 tensor [n, K]) for tokens idx against the fp32
    dequant-then-matmul oracle and the restated reference arithmetic (ref_bits, or computed)"""
    import numpy as np
    import torch

    from oracle import oracle as O

    xb = L.x[idx].view(torch.int16).numpy().view(np.uint16)
    ids, w = L.topk_ids[idx].numpy(), L.topk_weights[idx].numpy()
    fp32 = O.moe_fp32(xb, ids, w, L.type13, L.w13, L.type2, L.w2, L.inter)
    if ref_bits is None:
        ref_bits = O.moe_ref_bf16(xb, ids, w, L.type13, L.w13, L.type2, L.w2, L.inter)
    ref = O.bf16_to_f32(ref_bits)
    got = out_rows.float().cpu().numpy()
    return {"tokens_checked": int(len(idx)), "tokens": "spread evenly over the chunk",
            "rel_l2_vs_fp32": O.rel_l2(got, fp32), "rel_l2_vs_ref_arith": O.rel_l2(got, ref),
            "ref_arith_vs_fp32": O.rel_l2(ref, fp32), "bound_vs_fp32": 5e-3,
            "note": "the reference arithmetic (int8 q8_1 activations twice, bf16 intermediates) is itself "
                    "~1.2% from fp32, so no layer can be within 5e-3 of both"}


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args, rank):
    if rank != 0:
        return
    from kt_gguf_b200 import synth

    threads = host_threads()
    os.environ["OMP_NUM_THREADS"] = str(threads)
    import numpy as np
    import torch

    fn, kind = cpu_layer_fn()
    L = synth.make_layer(args.seed, **synth.CONFIGS[2])
    n = min(args.cpu_sample, L.x.shape[0])
    xb = L.x.view(torch.int16).numpy().view(np.uint16)
    ids = L.topk_ids.numpy()
    w = L.topk_weights.numpy()
    T = L.x.shape[0]

    def step(i):
        s = (i * n) % (T - n + 1)
        fn(xb[s:s + n], ids[s:s + n], w[s:s + n], L.type13, L.w13, L.type2, L.w2, L.inter)

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(args.warmup + i)
    dt = time.perf_counter() - t0
    value = n * args.steps / dt
    sample = f"{n} consecutive tokens of the 16K chunk per step (all their routes), extrapolated per token; {kind}"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 x gguf (q8_1 activations), fp32 accumulate",
        "data": "synthetic (seeded)",
        "config": {"workload": CONFIG_NAME, "tokens": T, "hidden": 2048, "inter": 512, "experts": 256, "top_k": 8,
                   "resident_experts": 64, "types": "Q4_K gate/up, Q6_K down", "device": "host CPU"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_b200(args, rank, world, local_rank):
    import numpy as np
    import torch

    from kt_gguf_b200 import _native as Nt
    from kt_gguf_b200 import kt_gguf_moe_multi as M
    from kt_gguf_b200 import synth

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    cfg = dict(synth.CONFIGS[2], tokens=args.tokens)
    L = synth.make_layer(args.seed + rank, **cfg)
    T, K, N = L.x.shape[0], cfg["hidden"], cfg["inter"]
    x = L.x.to(dev)
    w13 = torch.from_numpy(L.w13).to(dev)
    w2 = torch.from_numpy(L.w2).to(dev)
    ids = L.topk_ids.to(dev)
    wts = L.topk_weights.to(dev)
    S, k = w13.shape[0], ids.shape[1]
    lib = Nt.load()
    ws = Nt.workspace(lib.kt_moe_prefill_workspace_size(T, k, K, N, S), dev)
    out = torch.empty((T, K), dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)
    r_hot = int((L.topk_ids >= 0).sum())

    def step(timed=None):
        if timed is not None:
            timed[0][0].record(stream)
        Nt.check(lib.kt_moe_prefill_timed(Nt.ptr(x), T, K, N, Nt.ptr(ids), Nt.ptr(wts), k, Nt.ptr(w13), L.type13,
                                          Nt.ptr(w2), L.type2, 0, S, Nt.ptr(out), Nt.ptr(ws), ws.numel(), stream.cuda_stream,
                                          timed[1] if timed is not None else None), "kt_moe_prefill")

    # the clock sampler starts before the warm-up, so the GPU does not idle between the warm-up
    # and the timed steps
    uuid = torch.cuda.get_device_properties(dev).uuid
    sampler = ClockSampler(f"GPU-{uuid}") if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert Nt.workspace_status(ws) == Nt.KT_DEV_OK
    # per-stage times: a separate pass with stage events, steps queued back to back so the
    # device never waits for the host between stages (one event set per step)
    n_stage = max(4, min(20, args.steps))
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(n_stage)]
    for e in (e for es in evs for e in es):
        e.record(stream)  # torch only times events it has recorded; the library re-records them
    hs = [(ctypes.c_void_p * 4)(*[e.cuda_event for e in es[1:]]) for es in evs]
    for i in range(n_stage):
        step((evs[i], hs[i]))
    torch.cuda.synchronize()
    stage = [[evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(1, n_stage)] for j in range(4)]
    stage_ms = [statistics.median(s) for s in stage]

    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t_begin, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0 = time.time()
    t_begin.record(stream)
    for _ in range(args.steps):
        step()
    t_end.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    wall1 = time.time()
    ms = t_begin.elapsed_time(t_end)
    if dist:
        m = torch.tensor([ms], device=dev)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        ms = float(m.item())
    clocks = sampler.stop(wall0, wall1) if sampler else None
    assert Nt.workspace_status(ws) == Nt.KT_DEV_OK

    # end to end through the public API (kt_gguf_moe_multi.moe_prefill): every step copies its
    # inputs from pinned host memory and its output back. Steps are double-buffered over a
    # host-to-device stream, the compute stream and a device-to-host stream, so step i's
    # copies overlap steps i-1 / i+1's layer, the way a serving loop feeds prefill chunks.
    e2e = None
    if not args.no_e2e:
        x_h = L.x.pin_memory()
        ids_h = L.topk_ids.pin_memory()
        w_h = L.topk_weights.pin_memory()
        out_h = [torch.empty((T, K), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        xd = [torch.empty_like(x) for _ in range(2)]
        idd = [torch.empty_like(ids) for _ in range(2)]
        wd = [torch.empty_like(wts) for _ in range(2)]
        od = [torch.empty((T, K), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

        def e2e_run(n):
            done = [None, None]    # compute of the slot's previous step (its inputs are free)
            copied = [None, None]  # d2h of the slot's previous step (its output is free)
            for i in range(n):
                b = i % 2
                with torch.cuda.stream(h2d):
                    if done[b] is not None:
                        h2d.wait_event(done[b])
                    xd[b].copy_(x_h, non_blocking=True)
                    idd[b].copy_(ids_h, non_blocking=True)
                    wd[b].copy_(w_h, non_blocking=True)
                    ready = torch.cuda.Event()
                    ready.record(h2d)
                stream.wait_event(ready)
                if copied[b] is not None:
                    stream.wait_event(copied[b])
                M.moe_prefill(xd[b], w13, w2, idd[b], wd[b], L.type13, L.type2, N, workspace=ws, out=od[b])
                done[b] = torch.cuda.Event()
                done[b].record(stream)
                with torch.cuda.stream(d2h):
                    d2h.wait_event(done[b])
                    out_h[b].copy_(od[b], non_blocking=True)
                    copied[b] = torch.cuda.Event()
                    copied[b].record(d2h)
            for c in copied:
                if c is not None:
                    stream.wait_event(c)

        e2e_run(3)
        torch.cuda.synchronize()
        e_steps = max(8, args.steps // 4)
        if dist:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        h2d.wait_event(e0)
        d2h.wait_event(e0)
        e2e_run(e_steps)
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1)
        if dist:
            m = torch.tensor([e_ms], device=dev)
            dist.all_reduce(m, op=dist.ReduceOp.MAX)
            e_ms = float(m.item())
        assert torch.equal(out_h[(e_steps - 1) % 2], out.cpu()), "end-to-end output differs from the device run"
        e2e = {"value": world * T * e_steps / (e_ms * 1e-3), "unit": "tokens/s",
               "h2d_bytes_per_step": x_h.numel() * 2 + ids_h.numel() * 4 + w_h.numel() * 4,
               "d2h_bytes_per_step": out_h[0].numel() * 2,
               "overlap": "double-buffered: host-to-device, compute and device-to-host streams"}

    if rank == 0:
        hbm, tf_burst, tf_sust, peak_kind = load_peaks()
        flops_gate_up = 4.0 * K * N * r_hot
        flops_down = 2.0 * K * N * r_hot
        gate_up_tflops = flops_gate_up / (stage_ms[1] * 1e-3) / 1e12
        traffic = profile_traffic("prefill_gate_up_config2.txt")
        predq = int(lib.kt_moe_prefill_predequant(T, k, K, N, S))  # bit 0: gate/up weights, bit 1: down
        cpu = None
        idx = spread_tokens(T, args.cpu_sample)
        if world == 1 and not args.no_cpu_baseline:
            threads = host_threads()
            v, kind = cpu_baseline(L, idx, threads)
            macs = 3.0 * K * N * float((L.topk_ids[idx] >= 0).sum())
            cpu = {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                   "gmac_per_s": macs * v / len(idx) / 1e9,
                   "sample": f"{len(idx)} tokens spread evenly over the chunk (all their routes); {kind}"}
        parity = headline_parity(L, idx, out[torch.from_numpy(idx).to(dev)], None)
        value = world * T * args.steps / (ms * 1e-3)
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": ("bf16 (GGUF Q4_K gate/up and Q6_K down weights dequantized to bf16 once per call, "
                      "fp32 accumulate)" if predq == 3 else
                      "bf16 (GGUF Q4_K gate/up weights dequantized to bf16 once per call, Q6_K down weights "
                      "dequantized in-kernel, fp32 accumulate)" if predq else
                      "bf16 (GGUF Q4_K/Q6_K weights dequantized in-kernel, fp32 accumulate)"),
            "data": "synthetic (seeded)",
            "config": {"workload": CONFIG_NAME, "tokens_per_gpu": T, "hidden": K, "inter": N, "experts": 256,
                       "top_k": k, "resident_experts": S, "routed_to_resident": r_hot,
                       "types": "Q4_K gate/up, Q6_K down", "parallelism": f"token-parallel x{world} (replicated slots)",
                       "l2": "no flush: one step's working set (130 MB weights + 67 MB x + 0.66 GB H/Y) exceeds the 126 MB L2"},
            "stage_ms": {PASS_STAGE.get(predq, "permute"): stage_ms[0],
                         "gate_up_gemm": stage_ms[1], "down_gemm": stage_ms[2], "combine": stage_ms[3]},
            # the kernel runs for well under a second at the maximum SM clock (clocks below): the
            # burst cuBLAS figure is its ceiling; the sustained one applies under the power cap
            "roofline": {"bound": "tensor",
                         "kernel": ("kt_moe_gemm_kernel<gate/up, bf16 A by TMA> (the one-pass weight dequant is "
                                    "timed in stage_ms' first stage)" if predq else
                                    "kt_moe_gemm_kernel<Q4_K, gate/up>"),
                         "achieved": gate_up_tflops, "peak": tf_burst, "unit": "TFLOP/s",
                         "frac": gate_up_tflops / tf_burst, "peak_kind": f"{peak_kind} bf16 burst (cuBLAS)",
                         "frac_of_sustained": gate_up_tflops / tf_sust,
                         "traffic": traffic,
                         "down_gemm_tflops": flops_down / (stage_ms[2] * 1e-3) / 1e12,
                         "layer_tflops": (flops_gate_up + flops_down) * args.steps / (ms * 1e-3) / 1e12},
            "parity": parity,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": (6 + bin(predq).count("1")) * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def _ep_setup_config2(args, rank, world, dev):
    """Config 2: the 64 resident experts dealt hottest first in snake order; each rank its own
    16K-token chunk (same experts, different tokens)."""
    import torch

    from kt_gguf_b200 import ep as EP
    from kt_gguf_b200 import kt_gguf_moe_multi as M
    from kt_gguf_b200 import synth

    cfg = dict(synth.CONFIGS[2], tokens=args.tokens)
    L = synth.make_layer(args.seed, token_seed=args.seed + 1 + rank, **cfg)
    K, N = cfg["hidden"], cfg["inter"]
    S = L.w13.shape[0]
    owner, local = EP.snake_placement(S, world)
    mine = (owner == rank).nonzero().flatten()
    mine = mine[torch.argsort(local[mine])]
    w13_all = torch.from_numpy(L.w13).to(dev)
    w2_all = torch.from_numpy(L.w2).to(dev)
    w13 = w13_all[mine.to(dev)].contiguous()
    w2 = w2_all[mine.to(dev)].contiguous()
    x, ids, wts = L.x.to(dev), L.topk_ids.to(dev), L.topk_weights.to(dev)
    layer = EP.ExpertParallelMoE(owner, local, EP.prefill_expert_fn(w13, w2, L.type13, L.type2, N),
                                 chunks=args.ep_chunks)

    def ref_fn(n):  # the whole layer on this GPU (all 64 slots) for this rank's first n tokens
        return M.moe_prefill(x[:n].contiguous(), w13_all, w2_all, ids[:n].contiguous(), wts[:n].contiguous(),
                             L.type13, L.type2, N)

    r_all = int((L.topk_ids >= 0).sum())
    return dict(x=x, ids=ids, wts=wts, layer=layer, w13=w13, w2=w2, types=(L.type13, L.type2), K=K, N=N,
                ref_fn=ref_fn, flops=6.0 * K * N * r_all, metric=METRIC, workload=CONFIG_NAME,
                config={"experts": 256, "top_k": cfg["top_k"], "resident_experts": S,
                        "types": "Q4_K gate/up, Q6_K down",
                        "placement": "64 resident experts dealt hottest first in snake order"},
                host=(L.x, L.topk_ids, L.topk_weights))


def _ep_setup_config4(args, rank, world, dev):
    """Config 4: DeepSeek-V3-like layer, hidden 7168, expert intermediate 2048, 256 routed
    experts + 1 shared, grouped top-8 (8 groups, top-4 groups, sigmoid scores, renormalised,
    scale 2.5), Q4_K everywhere, 32768 tokens per rank; experts contiguous over the ranks.
    Weights: 16 distinct N(0,0.02) experts quantized to Q4_K, expert e holds copy e % 16 (the
    256 slots are distinct memory; generating 256 distinct experts on the host takes minutes)."""
    import numpy as np
    import torch

    from kt_gguf_b200 import ep as EP
    from kt_gguf_b200 import kernels as Kn
    from kt_gguf_b200 import kt_gguf_moe_multi as M
    from kt_gguf_b200 import synth

    K, N, E, k, T = 7168, 2048, 256, 8, args.tokens_c4
    rng = np.random.default_rng(args.seed)
    w13_16, w2_16 = synth.expert_weights(rng, 17, K, N, 12, 12)  # 16 routed + 1 shared
    w13_16 = torch.from_numpy(w13_16).to(dev)
    w2_16 = torch.from_numpy(w2_16).to(dev)
    owner, local = EP.contiguous_placement(E, world)
    per = E // world
    gids = torch.arange(rank * per, (rank + 1) * per)
    w13 = w13_16[(gids % 16).to(dev)].contiguous()
    w2 = w2_16[(gids % 16).to(dev)].contiguous()
    sw13, sw2 = w13_16[16:17].contiguous(), w2_16[16:17].contiguous()
    g = torch.Generator().manual_seed(args.seed + 1 + rank)
    x = torch.randn((T, K), generator=g).to(torch.bfloat16).to(dev)
    logits = torch.randn((T, E), generator=g).to(dev)
    bias = (torch.randn(E, generator=g) * 0.1).to(dev)
    wts, ids = Kn.topk_grouped(logits, bias, 8, 4, k, renormalize=True, scale=2.5)
    ones = torch.ones((T, 1), dtype=torch.float32, device=dev)
    zeros = torch.zeros((T, 1), dtype=torch.int32, device=dev)
    sh_ws = {}

    def shared_fn(xx):
        n = xx.shape[0]
        if "ws" not in sh_ws:
            from kt_gguf_b200 import _native as Nt

            sh_ws["ws"] = Nt.workspace(Nt.load().kt_moe_prefill_workspace_size(n, 1, K, N, 1), dev)
        return M.moe_prefill(xx, sw13, sw2, zeros[:n], ones[:n], 12, 12, N, workspace=sh_ws["ws"])

    layer = EP.ExpertParallelMoE(owner, local, EP.prefill_expert_fn(w13, w2, 12, 12, N), shared_fn=shared_fn,
                                 chunks=args.ep_chunks)

    def ref_fn(n):  # the whole layer on this GPU: expert e is copy e % 16, plus the shared expert
        r = M.moe_prefill(x[:n].contiguous(), w13_16[:16], w2_16[:16], (ids[:n] % 16).to(torch.int32).contiguous(),
                          wts[:n].contiguous(), 12, 12, N)
        return (r.float() + shared_fn(x[:n].contiguous()).float()).to(torch.bfloat16)

    return dict(x=x, ids=ids, wts=wts, layer=layer, w13=w13, w2=w2, types=(12, 12), K=K, N=N, ref_fn=ref_fn,
                flops=6.0 * K * N * (T * k + T), metric="DeepSeek-V3-like MoE layer tok/s @32K chunk",
                workload="deepseek-v3-like MoE layer (BASELINE configs[3])",
                config={"experts": E, "shared_experts": 1, "top_k": k, "routing": "grouped: 8 groups, top-4 groups",
                        "types": "Q4_K", "placement": "contiguous, %d experts per rank" % per,
                        "weights": "16 distinct experts, expert e holds copy e % 16"},
                host=(x.cpu(), ids.cpu(), wts.cpu()))


def run_ep(args, rank, world, local_rank, cfg_id=2):
    """Expert-parallel layer on `world` GPUs (kt_gguf_b200.ep): tokens go to the ranks owning
    their experts and the partial outputs come back by NCCL all-to-all. Each rank processes
    its own chunk, so per-rank work stays fixed as ranks are added ("weak")."""
    import datetime

    import torch
    import torch.distributed as dist

    from kt_gguf_b200 import _native as Nt

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        # NCCL prints its communicator set-up (ranks, transports) on stderr
        os.environ.setdefault("NCCL_DEBUG", "INFO")
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    st = (_ep_setup_config2 if cfg_id == 2 else _ep_setup_config4)(args, rank, world, dev)
    x, ids, wts, layer, w13, w2 = st["x"], st["ids"], st["wts"], st["layer"], st["w13"], st["w2"]
    K, N = st["K"], st["N"]
    T = x.shape[0]
    stream = torch.cuda.current_stream(dev)

    uuid = torch.cuda.get_device_properties(dev).uuid
    sampler = ClockSampler(f"GPU-{uuid}") if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    for _ in range(args.warmup):
        out = layer(x, ids, wts)
    torch.cuda.synchronize()
    n_chk = min(512, T)
    ref = st["ref_fn"](n_chk)
    err = float((out[:n_chk].float() - ref.float()).norm() / ref.float().norm())
    # phases of one call (events around dispatch, local experts, combine)
    p2p = world > 1 and layer.p2p and args.ep_chunks == 1
    ph, fine = [], []
    for _ in range(5):
        e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        if p2p:
            e8 = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
            layer._call_p2p(x, ids, wts, events=e8)
            torch.cuda.synchronize()
            fine.append([e8[j].elapsed_time(e8[j + 1]) for j in range(7)])
            e = [e8[0], e8[4], e8[5], e8[7]]
        else:
            e[0].record(stream)
            xr, ir, wr, plan = layer.dispatch(x, ids, wts)
            e[1].record(stream)
            yr = layer.expert_fn(xr, ir, wr)
            e[2].record(stream)
            layer.combine(yr, plan, T)
            e[3].record(stream)
        torch.cuda.synchronize()
        ph.append([e[j].elapsed_time(e[j + 1]) for j in range(3)])
    phases = [statistics.median(p[j] for p in ph) for j in range(3)]
    fine_ms = None
    if fine:
        names = ("plan", "count_all_gather", "dispatch_kernel", "barrier_rows_in_place", "local_experts",
                 "barrier_partials_in_place", "combine_kernel")
        fine_ms = {n: statistics.median(f[j] for f in fine) for j, n in enumerate(names)}
    if p2p:  # the received rows, from the exchange buffers (outside the timed region)
        n_recv = int(layer.peers.recv_total.item())
        xr, ir, wr = layer.peers.x[:n_recv], layer.peers.ids[:n_recv], layer.peers.w[:n_recv]
    n_recv = int(xr.shape[0])
    # local GEMM stages on the received rows (for the roofline)
    lib = Nt.load()
    ws = Nt.workspace(lib.kt_moe_prefill_workspace_size(n_recv, ir.shape[1], K, N, w13.shape[0]), dev)
    yl = torch.empty((n_recv, K), dtype=torch.bfloat16, device=dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(6)]
    for ee in (ee for es in evs for ee in es):
        ee.record(stream)
    hs = [(ctypes.c_void_p * 4)(*[ee.cuda_event for ee in es[1:]]) for es in evs]
    for i in range(6):
        evs[i][0].record(stream)
        Nt.check(lib.kt_moe_prefill_timed(Nt.ptr(xr), n_recv, K, N, Nt.ptr(ir), Nt.ptr(wr), ir.shape[1], Nt.ptr(w13),
                                          st["types"][0], Nt.ptr(w2), st["types"][1], 0, w13.shape[0], Nt.ptr(yl),
                                          Nt.ptr(ws), ws.numel(), stream.cuda_stream, hs[i]), "kt_moe_prefill")
    torch.cuda.synchronize()
    stage_ms = [statistics.median(evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(1, 6)) for j in range(4)]
    r_local = int((ir >= 0).sum())
    predq_ep = int(lib.kt_moe_prefill_predequant(n_recv, ir.shape[1], K, N, w13.shape[0]))  # the one-pass dequant bits
    for _ in range(2):  # back to the exchange after the stage pass (untimed)
        out = layer(x, ids, wts)

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0 = time.time()
    t0.record(stream)
    for _ in range(args.steps):
        out = layer(x, ids, wts)
    t1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    wall1 = time.time()
    m = torch.tensor([t0.elapsed_time(t1)], device=dev)
    if world > 1:
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
    ms = float(m.item())
    clocks = sampler.stop(wall0, wall1) if sampler else None

    e2e = None
    if not args.no_e2e:
        x_h, ids_h, w_h = (t.pin_memory() for t in st["host"])
        out_h = torch.empty((T, K), dtype=torch.bfloat16).pin_memory()

        def e2e_step():
            o = layer(x_h.to(dev, non_blocking=True), ids_h.to(dev, non_blocking=True), w_h.to(dev, non_blocking=True))
            out_h.copy_(o, non_blocking=True)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        e_steps = max(5, args.steps // 4)
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        me = torch.tensor([e0.elapsed_time(e1)], device=dev)
        if world > 1:
            dist.all_reduce(me, op=dist.ReduceOp.MAX)
        e2e = {"value": world * T * e_steps / (float(me.item()) * 1e-3), "unit": "tokens/s",
               "h2d_bytes_per_step": x_h.numel() * 2 + ids_h.numel() * 4 + w_h.numel() * 4,
               "d2h_bytes_per_step": out_h.numel() * 2, "overlap": "none (sequential copies around each call)"}
    # per-rank figures: check error, rows received, and the unpipelined phases (the local
    # experts' time differs by rank with the load; the max-min spread is time the exchange
    # spends waiting for the slowest rank)
    mine = torch.tensor([err, float(n_recv), phases[0], phases[1], phases[2]], device=dev)
    every = [mine]
    if world > 1:
        every = [torch.zeros(5, device=dev) for _ in range(world)]
        dist.all_gather(every, mine)
    every = [v.tolist() for v in every]
    if rank == 0:
        hbm, tf_burst, tf_sust, peak_kind = load_peaks()
        tf13 = 4.0 * K * N * r_local / (stage_ms[1] * 1e-3) / 1e12
        line = {
            "metric": st["metric"], "value": world * T * args.steps / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": ("bf16 (GGUF weights dequantized to bf16 once per call, fp32 accumulate)" if predq_ep == 3 else
                      "bf16 (GGUF gate/up weights dequantized to bf16 once per call, down in-kernel, fp32 accumulate)"
                      if predq_ep else "bf16 (GGUF weights dequantized in-kernel, fp32 accumulate)"),
            "data": "synthetic (seeded)",
            "config": dict({"workload": st["workload"], "tokens_per_gpu": T, "hidden": K, "inter": N,
                            "parallelism": f"ep{world}",
                            "l2": "no flush: one step's working set exceeds the 126 MB L2"}, **st["config"]),
            "layer_tflops": world * st["flops"] * args.steps / (ms * 1e-3) / 1e12,
            "ep": {"phase_ms_unpipelined": {"dispatch": phases[0], "local_experts": phases[1], "combine": phases[2]},
                   "exchange_ms_rank0": fine_ms,
                   "local_experts_ms_per_rank": [v[3] for v in every],
                   "local_experts_imbalance_ms": max(v[3] for v in every) - min(v[3] for v in every),
                   "dispatch_ms_per_rank": [v[2] for v in every],
                   "combine_ms_per_rank": [v[4] for v in every],
                   "chunks": args.ep_chunks,
                   "rows_received_per_rank": [int(v[1]) for v in every],
                   "check_rel_l2_vs_single_gpu_layer": max(v[0] for v in every),
                   "collective": ("peer memory over NVLink: the dispatch kernel stores rows into the other ranks' "
                                  "receive buffers, the combine kernel loads the partials from their output buffers "
                                  "(CUDA IPC); NCCL only for an all-gather of the row counts and two one-word "
                                  "all-reduce barriers") if p2p else
                                 "torch.distributed.all_to_all_single over NCCL (counts, rows, metadata; partials back)",
                   "nccl": {"version": ".".join(map(str, torch.cuda.nccl.version())), "ranks": world,
                            "backend": dist.get_backend() if world > 1 else None}},
            "stage_ms_local": {PASS_STAGE.get(predq_ep, "permute"): stage_ms[0],
                               "gate_up_gemm": stage_ms[1], "down_gemm": stage_ms[2], "combine": stage_ms[3]},
            "roofline": {"bound": "tensor", "kernel": "kt_moe_gemm_kernel<Q4_K, gate/up> (rank 0's received rows)",
                         "achieved": tf13, "peak": tf_burst, "unit": "TFLOP/s", "frac": tf13 / tf_burst,
                         "peak_kind": f"{peak_kind} bf16 burst (cuBLAS)",
                         "traffic": None},
            "cpu_baseline": None,
            "e2e": e2e,
            # per call: the plan (3 kernels), the row packing, the layer (6), the combine of the
            # partials; one rank skips the exchange and runs the layer alone
            "gpu_launches": ((11 if world > 1 else 6) + bin(predq_ep).count("1")) * args.steps * args.ep_chunks,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        layer.close()
        dist.barrier()
        dist.destroy_process_group()


def run_config5(args):
    """Config 5: a 48-layer prefill of a 65536-token prompt in 16384-token chunks. Each layer
    runs one dense bf16 projection [4096 x 2048] (cuBLAS through torch.matmul) and the
    config-2 MoE layer (tcgen05 path, x += moe(x)); the dense weights live in pinned host
    memory and come back one layer ahead on a side stream (kt_gguf_b200.lend.LayerStreamer:
    two device slots, event-ordered copies). Reported: tokens/s of the whole prompt, the H2D
    rate of the copies, the fraction of copy time hidden under compute, and the same pass
    with the dense weights resident (the cost of streaming). One expert set serves all 48
    layers (per-layer work and bytes are those of distinct layers)."""
    import torch

    from kt_gguf_b200 import _native as Nt
    from kt_gguf_b200 import kt_gguf_moe_multi as M
    from kt_gguf_b200 import lend
    from kt_gguf_b200 import synth

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n_layers, prompt, chunk, dense_rows = 48, 65536, 16384, 4096
    cfg = dict(synth.CONFIGS[2], tokens=prompt)
    L = synth.make_layer(args.seed, **cfg)
    K, N = cfg["hidden"], cfg["inter"]
    w13, w2 = torch.from_numpy(L.w13).to(dev), torch.from_numpy(L.w2).to(dev)
    x_all = L.x.to(dev)
    ids_all, w_all = L.topk_ids.to(dev), L.topk_weights.to(dev)
    g = torch.Generator().manual_seed(args.seed + 5)
    host = [(torch.randn((dense_rows, K), generator=g) * 0.02).to(torch.bfloat16).pin_memory() for _ in range(n_layers)]
    resident = [h.to(dev) for h in host]
    lib = Nt.load()
    ws = Nt.workspace(lib.kt_moe_prefill_workspace_size(chunk, ids_all.shape[1], K, N, w13.shape[0]), dev)
    stream = torch.cuda.current_stream(dev)

    def prompt_pass(weights_for):
        for c0 in range(0, prompt, chunk):
            x = x_all[c0:c0 + chunk].clone()
            ids, wts = ids_all[c0:c0 + chunk].contiguous(), w_all[c0:c0 + chunk].contiguous()
            for li in range(n_layers):
                wd = weights_for(li)
                h = torch.matmul(x, wd.t())  # the layer's dense projection
                del h
                x += M.moe_prefill(x, w13, w2, ids, wts, L.type13, L.type2, N, workspace=ws)
            if hasattr(weights_for, "finish"):
                weights_for.finish()

    class Streamed:
        def __init__(self, timing):
            self.s = lend.LayerStreamer(host, dev, timing=timing)

        def __call__(self, li):
            return self.s.enter(li)

        def finish(self):
            self.s.finish()

    def timed(fn):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    warm = Streamed(False)
    prompt_pass(warm)  # warm-up (cuBLAS heuristics, library state)
    ms_res = timed(lambda: prompt_pass(lambda li: resident[li]))
    sw = Streamed(True)
    ms_str = timed(lambda: prompt_pass(sw))
    stt = sw.s.stats()
    line = {"metric": "config 5 prompt", "value": prompt / (ms_str * 1e-3), "unit": "tokens/s",
            "ms_prompt_streamed": ms_str, "ms_prompt_resident": ms_res,
            "streaming_overhead_frac": ms_str / ms_res - 1.0,
            "lend": {"copies": stt["copies"], "bytes": stt["bytes"], "h2d_GBps": stt["h2d_GBps"],
                     "copy_ms": stt["copy_ms"], "compute_wait_ms": stt["wait_ms"], "hidden_frac": stt["hidden_frac"]},
            "config": {"workload": "48-layer lend pipeline (BASELINE configs[4])", "layers": n_layers,
                       "prompt_tokens": prompt, "chunk": chunk, "dense_weight": [dense_rows, K],
                       "moe": "config 2 layer (Q4_K/Q6_K, 64 resident experts), one expert set for all layers"},
            "data": "synthetic (seeded)"}
    print(json.dumps(line), flush=True)


def run_stream(args):
    """Config 2 with its non-resident experts streamed instead of left to the CPU: the 64 hottest
    experts stay in their slots (tcgen05 prefill layer), the other 192 come from pinned host
    banks in groups, copied on a side stream while the previous group computes
    (kt_stream_prefill_gguf.KTStreamPrefillGGUF, the reference's KT_GPU_STREAM_PREFILL path).
    A step is the GPU side of one 16K-token chunk: resident layer + streamed groups + their sum.
    Reported: tokens/s, the H2D rate of the staged bytes over the step, and a plain pinned
    H2D copy of the same bytes (no compute) measured in this run as the bound (PCIe)."""
    from types import SimpleNamespace

    import numpy as np
    import torch

    from kt_gguf_b200 import _native as Nt
    from kt_gguf_b200 import kt_gguf_moe_multi as M
    from kt_gguf_b200 import kt_stream_prefill_gguf as SP
    from kt_gguf_b200 import synth

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = dict(synth.CONFIGS[2], tokens=args.tokens)
    n_res = cfg.pop("n_hot")
    E = cfg["n_experts"]
    # every expert with weights, physical order = hotness order: slots 0..63 are the resident
    # experts and the router's physical ids index the bank directly
    L = synth.make_layer(args.seed, n_hot=E, **cfg)
    K, Nn = cfg["hidden"], cfg["inter"]

    class Reader:
        def __init__(self):
            self.E = E

        def types(self, li):
            return (L.type13, L.type13, L.type2)

        def slice(self, li, proj, n, rank, experts):
            e = experts.numpy()
            v = {"gate": L.w13[e, :n], "up": L.w13[e, n:], "down": L.w2[e]}[proj]
            return torch.from_numpy(np.ascontiguousarray(v))

    method = SimpleNamespace(reader=Reader(), rank=0, world=1, N=Nn, K=K, num_gpu_experts=n_res,
                             kt_config=SimpleNamespace(layer_idx=0), streams_hot_experts=False)
    sp = SP.KTStreamPrefillGGUF(method, group_size=args.group or None)
    w13r, w2r = torch.from_numpy(L.w13[:n_res]).to(dev), torch.from_numpy(L.w2[:n_res]).to(dev)
    x, ids, wts = L.x.to(dev), L.topk_ids.to(dev), L.topk_weights.to(dev)
    slot_ids = torch.where(ids < n_res, ids, torch.full_like(ids, -1))
    d = SimpleNamespace(hidden_states=x, topk_output=SimpleNamespace(topk_weights=wts))
    lib = Nt.load()
    ws = Nt.workspace(lib.kt_moe_prefill_workspace_size(args.tokens, ids.shape[1], K, Nn, n_res), dev)
    stream = torch.cuda.current_stream(dev)

    def hot_only():
        return M.moe_prefill(x, w13r, w2r, slot_ids, wts, L.type13, L.type2, Nn, workspace=ws)

    def step():
        return hot_only().add_(sp.run(method, None, d, ids))

    def timed(fn, n):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    for _ in range(max(3, args.warmup)):  # builds the bank, library state
        step()
    steps = max(1, min(args.steps, 20))
    b0 = sp.bytes_staged
    ms = timed(step, steps)
    bytes_step = (sp.bytes_staged - b0) / steps
    ms_hot = timed(hot_only, steps)
    # the bound: the same bytes as plain pinned H2D copies, no compute
    banks = sp._bank(0)
    dst = [torch.empty(b[n_res:].numel(), dtype=torch.uint8, device=dev) for b in banks]

    def copy_only():
        for b, t in zip(banks, dst):
            t.copy_(b[n_res:].reshape(-1), non_blocking=True)

    ms_copy = timed(copy_only, 5)
    peak = bytes_step / (ms_copy * 1e-3) / 1e9
    got = bytes_step / (ms * 1e-3) / 1e9
    line = {"metric": "config 2 streamed prefill", "value": args.tokens / (ms * 1e-3), "unit": "tokens/s",
            "ms_per_step": ms, "ms_resident_only": ms_hot, "steps": steps,
            "stream": {"experts": E - n_res, "group": sp.G, "groups": len(sp.groups(n_res)),
                       "bytes_per_step": bytes_step, "h2d_GBps": got, "h2d_copy_only_GBps": peak,
                       "frac_of_copy_only": got / peak, "ms_copy_only": ms_copy},
            "config": {"workload": "config 2 (BASELINE configs[1]) with the 192 non-resident experts streamed",
                       "tokens": args.tokens, "resident_experts": n_res, "streamed_experts": E - n_res},
            "data": "synthetic (seeded)"}
    print(json.dumps(line), flush=True)


def _gemv_call(lib, Nt, x, w, ids, top_k, qtype, rows, tokens, y, ws, stream):
    Nt.check(lib.kt_moe_a8_vec_multi(Nt.ptr(x), Nt.dtype_code(x), tokens, x.shape[1], Nt.ptr(w), 0, w.shape[0],
                                     Nt.ptr(ids), top_k, qtype, rows, Nt.ptr(y), Nt.ptr(ws), ws.numel(), stream),
             "kt_moe_a8_vec_multi")


def run_sweep(args, cfg_id):
    """Decode GEMV points (HBM roofline, L2 flushed before every call) and prefill points
    (tensor roofline) on one config's layer: config 3 (IQ3_S, 512 experts all resident,
    top-10) or config 2 (Q4_K/Q6_K, 64 of 256 experts resident, top-8)."""
    import numpy as np
    import torch

    from kt_gguf_b200 import _native as Nt
    from kt_gguf_b200 import kernels as Kn
    from kt_gguf_b200 import kt_gguf_moe_multi as M
    from kt_gguf_b200 import synth

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = synth.CONFIGS[cfg_id]
    L = synth.make_layer(args.seed, **cfg)
    K, N, k = cfg["hidden"], cfg["inter"], cfg["top_k"]
    E = L.w13.shape[0]  # resident slots
    t13, t2 = L.type13, L.type2
    w13 = torch.from_numpy(L.w13).to(dev)
    w2 = torch.from_numpy(L.w2).to(dev)
    x_all = L.x.to(dev)
    ids_all = L.topk_ids.to(dev)
    w_all = L.topk_weights.to(dev)
    lib = Nt.load()
    stream = torch.cuda.current_stream(dev)
    hbm, tf_burst, tf_sust, peak_kind = load_peaks()
    b13 = w13.shape[1] * w13.shape[2]  # bytes of one expert's gate/up rows
    b2 = w2.shape[1] * w2.shape[2]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # 2x the L2
    names = {3: "flash-next-like IQ3_S MoE layer (BASELINE configs[2])", 2: CONFIG_NAME}
    base = {"metric": f"config {cfg_id} point", "config": {"workload": names[cfg_id], "hidden": K, "inter": N,
                                                           "experts": cfg["n_experts"], "resident": E, "top_k": k,
                                                           "types": f"ggml {t13} gate/up, {t2} down"},
            "data": "synthetic (seeded)"}
    iters = max(20, min(args.steps, 200))
    m_list = [int(v) for v in args.m_list.split(",") if v]
    for Mtok in [m for m in m_list if m < 128]:
        ws13 = Nt.workspace(lib.kt_moe_a8_vec_workspace_size(Mtok, K, Mtok * k, E), dev)
        ws2 = Nt.workspace(lib.kt_moe_a8_vec_workspace_size(Mtok * k, N, Mtok * k, E), dev)
        h13 = torch.empty((Mtok * k, 2 * N), dtype=torch.bfloat16, device=dev)
        y = torch.empty((Mtok * k, K), dtype=torch.bfloat16, device=dev)
        s13, s2, tl, uniq = [], [], [], []
        for it in range(args.warmup + iters):
            r0 = (it * Mtok) % (x_all.shape[0] - Mtok)  # a different window each call: different experts
            x = x_all[r0:r0 + Mtok]
            ids = ids_all[r0:r0 + Mtok].reshape(-1).contiguous()
            flush.zero_()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            ev[0].record(stream)
            _gemv_call(lib, Nt, x, w13, ids, k, t13, 2 * N, Mtok, h13, ws13, stream.cuda_stream)
            ev[1].record(stream)
            h = Kn.silu_and_mul(h13)
            ev[2].record(stream)
            _gemv_call(lib, Nt, h, w2, ids, 1, t2, K, Mtok * k, y, ws2, stream.cuda_stream)
            ev[3].record(stream)
            Kn.combine(y.view(Mtok, k, K), w_all[r0:r0 + Mtok])
            torch.cuda.synchronize()
            if it >= args.warmup:
                s13.append(ev[0].elapsed_time(ev[1]))
                s2.append(ev[2].elapsed_time(ev[3]))
                tl.append(ev[0].elapsed_time(ev[3]))
                u_ids = torch.unique(ids)
                uniq.append(int((u_ids >= 0).sum()))
        u = statistics.mean(uniq)
        g13 = u * b13 / (statistics.median(s13) * 1e-3) / 1e9
        g2 = u * b2 / (statistics.median(s2) * 1e-3) / 1e9
        line = dict(base, path="decode GEMV (q8_1 x GGUF, reference arithmetic)", M=Mtok,
                    unique_experts=u, ms_gate_up=statistics.median(s13), ms_down=statistics.median(s2),
                    ms_layer_without_combine=statistics.median(tl),
                    roofline={"bound": "hbm", "gate_up_GBps": g13, "down_GBps": g2, "peak": hbm, "unit": "GB/s",
                              "gate_up_frac": g13 / hbm, "down_frac": g2 / hbm, "peak_kind": f"{peak_kind} copy",
                              "bytes": "unique experts' GGUF bytes per call (gate/up %d B, down %d B per expert)" % (b13, b2)},
                    l2="256 MB buffer written before every call", iters=iters)
        print(json.dumps(line), flush=True)
    for Mtok in [m for m in m_list if m >= 128]:
        x = x_all[:Mtok].contiguous()
        ids = ids_all[:Mtok].contiguous()
        wts = w_all[:Mtok].contiguous()
        ws = Nt.workspace(lib.kt_moe_prefill_workspace_size(Mtok, k, K, N, E), dev)
        out = torch.empty((Mtok, K), dtype=torch.bfloat16, device=dev)
        n = max(4, min(20, args.steps))
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.warmup + n)]
        for e in (e for es in evs for e in es):
            e.record(stream)
        hs = [(ctypes.c_void_p * 4)(*[e.cuda_event for e in es[1:]]) for es in evs]
        for i in range(args.warmup + n):
            evs[i][0].record(stream)
            Nt.check(lib.kt_moe_prefill_timed(Nt.ptr(x), Mtok, K, N, Nt.ptr(ids), Nt.ptr(wts), k, Nt.ptr(w13), t13,
                                              Nt.ptr(w2), t2, 0, E, Nt.ptr(out), Nt.ptr(ws), ws.numel(),
                                              stream.cuda_stream, hs[i]), "kt_moe_prefill")
        torch.cuda.synchronize()
        assert Nt.workspace_status(ws) == Nt.KT_DEV_OK
        st = [statistics.median(evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(args.warmup, args.warmup + n))
              for j in range(4)]
        R = int((L.topk_ids[:Mtok] >= 0).sum())  # resident routes
        tf13 = 4.0 * K * N * R / (st[1] * 1e-3) / 1e12
        tf2 = 2.0 * K * N * R / (st[2] * 1e-3) / 1e12
        line = dict(base, path="prefill (tcgen05 GEMMs)", M=Mtok, value=Mtok / (sum(st) * 1e-3), unit="tokens/s",
                    stage_ms={"permute": st[0], "gate_up_gemm": st[1], "down_gemm": st[2], "combine": st[3]},
                    roofline={"bound": "tensor", "gate_up_tflops": tf13, "down_tflops": tf2, "peak": tf_burst,
                              "unit": "TFLOP/s", "gate_up_frac": tf13 / tf_burst, "down_frac": tf2 / tf_burst,
                              "peak_kind": f"{peak_kind} bf16 burst (cuBLAS)"})
        print(json.dumps(line), flush=True)


def run_config1(args):
    """Q8_0, 16 experts top-4, 256 tokens: GPU layer, CPU baseline on the whole chunk, parity."""
    import numpy as np
    import torch

    from kt_gguf_b200 import _native as Nt
    from kt_gguf_b200 import kt_gguf_moe_multi as M
    from kt_gguf_b200 import synth
    from oracle import oracle as O

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = synth.CONFIGS[1]
    L = synth.make_layer(args.seed, **cfg)
    K, N, k = cfg["hidden"], cfg["inter"], cfg["top_k"]
    x, ids, wts = L.x.to(dev), L.topk_ids.to(dev), L.topk_weights.to(dev)
    w13, w2 = torch.from_numpy(L.w13).to(dev), torch.from_numpy(L.w2).to(dev)
    lib = Nt.load()
    T = x.shape[0]
    ws = Nt.workspace(lib.kt_moe_prefill_workspace_size(T, k, K, N, w13.shape[0]), dev)
    out = torch.empty((T, K), dtype=torch.bfloat16, device=dev)
    for _ in range(args.warmup):
        M.moe_prefill(x, w13, w2, ids, wts, 8, 8, N, out=out, workspace=ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        M.moe_prefill(x, w13, w2, ids, wts, 8, 8, N, out=out, workspace=ws)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    xb = L.x.view(torch.int16).numpy().view(np.uint16)
    want = O.moe_fp32(xb, L.topk_ids.numpy(), L.topk_weights.numpy(), 8, L.w13, 8, L.w2, N)
    err = O.rel_l2(out.float().cpu().numpy(), want)
    threads = host_threads()
    os.environ["OMP_NUM_THREADS"] = str(threads)
    fn, kind = cpu_layer_fn()
    fn(xb[:8], L.topk_ids.numpy()[:8], L.topk_weights.numpy()[:8], 8, L.w13, 8, L.w2, N)
    t = time.perf_counter()
    fn(xb, L.topk_ids.numpy(), L.topk_weights.numpy(), 8, L.w13, 8, L.w2, N)
    cpu_s = time.perf_counter() - t
    line = {"metric": "config 1 layer", "value": T / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms,
            "steps": args.steps, "config": {"workload": "Q8_0 MoE layer (BASELINE configs[0])", "tokens": T,
                                             "hidden": K, "inter": N, "experts": cfg["n_experts"], "top_k": k},
            "rel_l2_vs_fp32_oracle": err, "tolerance": 5e-3,
            "cpu_baseline": {"value": T / cpu_s, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"the whole 256-token chunk; {kind}"},
            "data": "synthetic (seeded)"}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.config == 3 or (args.config == 2 and args.sweep):
        run_sweep(args, args.config)
        return
    if args.config == 1:
        run_config1(args)
        return
    if args.config == 4:
        run_ep(args, rank, world, local_rank, cfg_id=4)
        return
    if args.config == 5:
        run_config5(args)
        return
    if args.ep or (world > 1 and not args.replicas):
        run_ep(args, rank, world, local_rank)
        return
    if args.stream:
        run_stream(args)
        return
    run_b200(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
