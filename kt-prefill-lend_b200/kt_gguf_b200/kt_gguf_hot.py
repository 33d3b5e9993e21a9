"""Hot GPU experts straight from a GGUF, for the KT hybrid — B200 (sm_100a) implementation.

Drop-in for sglang.srt.layers.moe.kt_gguf_hot (hot/kt_gguf_hot.py): the GPU slots
0..num_gpu_experts-1 hold this rank's slice of each hot expert's raw GGUF blocks, in the
reference's layout:
  w13_qweight  uint8 [E_gpu, 2N, row_bytes(K, gate/up type)]   rows [gate; up]
  w2_qweight   uint8 [E_gpu, K,  row_bytes(N, down type)]
(hot/kt_gguf_hot.py:17-20). Ids < 0 (experts on the CPU) contribute nothing.

`apply` runs, per MoE layer call:
- bf16 chunks of at least PREFILL_MIN tokens: the tcgen05 prefill layer
  (kt_gguf_moe_multi.moe_prefill: gate/up GEMM with SwiGLU, down GEMM, fp32 weighted sum),
  in place of the reference's streamed prefill (dequant to bf16 + CUTLASS fused MoE);
- smaller windows (decode, MTP verify, short extends): the q8_1 GEMV
  (moe_a8_vec_multi, bit-identical to the reference kernel), silu_and_mul, the GEMV on the
  down weights and the reference combine (hot/kt_gguf_hot.py:240-304).
With KV-lent slots (layer.kt_kv_ptr13 / kt_kv_ptr2) both paths read the weights through the
per-slot pointer tables.

GGUF types with B200 kernels: the prefill layer takes Q8_0 (8), Q4_K (12), Q6_K (14) and
IQ3_S (21); the GEMV also Q4_0/Q4_1/Q5_0/Q5_1/IQ4_NL, Q2_K/Q3_K/Q5_K/IQ4_XS,
IQ2_XXS/IQ2_XS/IQ2_S/IQ3_XXS/IQ1_S/IQ1_M and the reference's Q2_0 (42); other types raise at
construction. As in the reference
(hot/kt_gguf_hot.py:21-25, 180-190), Q2_0 downs stay 2-bit on the GPU and their layers run
the GEMV at every length; KT_GGUF_Q2_NATIVE=0 repacks them losslessly into Q8_0 instead
(q2_0_to_q8_0), which the prefill layer takes.
"""
import os
import time
from typing import Dict, Tuple

import numpy as np
import torch
from torch.nn import Parameter

from . import kernels as _k
from . import kt_gguf_moe_multi as _multi

try:  # the serving tree's types when this module is installed into it
    from sglang.srt.layers.quantization.base_config import FusedMoEMethodBase
except ImportError:  # standalone use: the method only needs a plain base class
    FusedMoEMethodBase = object

try:
    from sglang.srt.layers.moe.token_dispatcher import StandardCombineInput
except ImportError:
    from dataclasses import dataclass

    @dataclass
    class StandardCombineInput:  # same field as SGLang's
        hidden_states: torch.Tensor

# The hot method's fused weighting + sum over top_k is bit-identical to out.mul_(w) + moe_sum
# (hot/kt_gguf_hot.py:37-38); the B200 combine kernel implements it at every token count.
FUSED_COMBINE = os.environ.get("KT_HOT_FUSED_COMBINE", "1") == "1"
# bf16 chunks from this many tokens go through the tcgen05 prefill layer
PREFILL_MIN = int(os.environ.get("KT_B200_PREFILL_MIN", "128"))
PREFILL_ON_GPU = os.environ.get("KT_B200_PREFILL", "1") == "1"

GGML_Q8_0 = 8
GGML_Q2_0 = 42
# ggml type -> (block elements, block bytes), the reference's table (hot/kt_gguf_hot.py:76-80)
# (19 is IQ1_S's 50-byte block here, as in the reference kernel's block_iq1_s; the reference's
# Python table gives it 74 bytes, IQ2_XS's size, and lacks 17 and 29)
BLOCK_INFO = {
    2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 10: (256, 84), 11: (256, 110),
    12: (256, 144), 13: (256, 176), 14: (256, 210),
    16: (256, 66), 17: (256, 74), 19: (256, 50), 20: (32, 18), 21: (256, 110), 22: (256, 82), 23: (256, 136),
    18: (256, 98), 29: (256, 56), 42: (64, 18),
}
# types with a B200 kernel (the reference's MMVQ_TYPES lists every sgl-kernel MMVQ type, which
# excludes its own Q2_0: that one is allowed through q2_native)
MMVQ_TYPES = set(_multi.SUPPORTED_TYPES) - {GGML_Q2_0}


def _log(msg):
    print(f"[kt-gguf-hot {time.strftime('%H:%M:%S')}] {msg}", flush=True)


def _row_bytes(cols: int, t: int) -> int:
    blck, ts = BLOCK_INFO[t]
    if cols % blck:
        raise ValueError(f"{cols} columns are not a multiple of the type {t} block ({blck})")
    return cols // blck * ts


def q2_0_to_q8_0(raw: torch.Tensor) -> torch.Tensor:
    """[..., n_blocks*18] Q2_0 bytes -> [..., n_blocks*2*34] Q8_0 bytes, exact: each 64-value
    block (fp16 d, 2-bit codes c, value = d*(c-1)) becomes two 32-value Q8_0 blocks with the
    same d and the codes minus one as int8."""
    shape = raw.shape[:-1]
    b = raw.reshape(-1, 18).cpu().numpy()
    n = b.shape[0]
    codes = ((b[:, 2:, None] >> np.array([0, 2, 4, 6], dtype=np.uint8)) & 3).reshape(n, 64).astype(np.int8) - 1
    out = np.empty((n, 2, 34), dtype=np.uint8)
    out[:, :, :2] = b[:, None, :2]
    out[:, :, 2:] = codes.reshape(n, 2, 32).view(np.uint8)
    return torch.from_numpy(out.reshape(*shape, -1))


def _combine(out: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """out [T, top_k, K] (the routes' rows), w [T, top_k]: sum_k bf16(out * bf16(w)) in fp32,
    rounded once (hot/kt_gguf_hot.py:58-71)."""
    return _k.combine(out, w)


class _GGUFExperts:
    """One GGUF reader shared by all layers of a rank (kt_kernel's GGUFLoader, as in the
    reference); slices return raw expert bytes in the slot layout."""

    def __init__(self, path: str):
        from kt_kernel.utils.loader import GGUFLoader  # the reference's loader, from its CPU library

        self.loader = GGUFLoader(path)
        cfg = self.loader.get_model_config()
        self.E = int(cfg["num_experts"])
        self.inter = int(cfg["moe_intermediate_size"])
        self.K = int(cfg["hidden_size"])

    def _raw(self, name: str) -> Tuple[torch.Tensor, int]:
        import warnings

        info = self.loader.tensor_info[name]
        t = int(info["dtype"])
        blck, ts = BLOCK_INFO[t]
        n_bytes = int(info["n_elements"]) // blck * ts
        mm = self.loader.file_data_map[self.loader.tensor_file_map[name]]
        raw = np.frombuffer(mm, dtype=np.uint8, count=n_bytes, offset=int(info["offset"]))
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")  # read-only mapping, only copied from
            return torch.from_numpy(raw), t

    def types(self, layer_idx: int) -> Tuple[int, int, int]:
        return tuple(int(self.loader.get_ggml_type(f"blk.{layer_idx}.ffn_{p}_exps.weight")) for p in ("gate", "up", "down"))

    def slice(self, layer_idx: int, proj: str, N: int, rank: int, experts: torch.Tensor) -> torch.Tensor:
        """This rank's tensor-parallel part of the given experts: rows [N*rank, N*(rank+1)) of
        gate/up, the matching block-aligned columns of down. uint8 [len(experts), rows, bytes]."""
        data, t = self._raw(f"blk.{layer_idx}.ffn_{proj}_exps.weight")
        blck, ts = BLOCK_INFO[t]
        if proj != "down":
            v = data.view(self.E, self.inter, (self.K // blck) * ts)[experts, N * rank:N * (rank + 1), :]
        else:
            v = data.view(self.E, self.K, self.inter // blck, ts)[experts, :, (N * rank) // blck:(N * (rank + 1)) // blck, :]
            v = v.reshape(len(experts), self.K, -1)
        return v.contiguous()


_readers: Dict[str, object] = {}


def _reader(path: str):
    r = _readers.get(path)
    if r is None:
        r = _readers[path] = _GGUFExperts(path)
    return r


class KTGGUFHotExpertsMethod(FusedMoEMethodBase):
    """GPU-expert method the KT wrapper wraps when the experts are a GGUF."""

    # the reference skips this method at streamed-prefill sizes (its kernel is a decode
    # kernel); with the B200 prefill layer the method serves prefill chunks itself
    streams_hot_experts = not PREFILL_ON_GPU

    def __init__(self, kt_config, layer):
        self.kt_config = kt_config
        self.num_gpu_experts = kt_config.num_gpu_experts
        self.reader = _reader(kt_config.weight_path)
        self.rank, self.world = layer.moe_tp_rank, layer.moe_tp_size
        self.types = self.reader.types(kt_config.layer_idx)
        if self.types[0] != self.types[1]:
            raise RuntimeError(f"layer {kt_config.layer_idx}: gate {self.types[0]} and up {self.types[1]} differ")
        self.type13 = self.types[0]
        # Q2_0 downs stay 2-bit on the GPU (KT_GGUF_Q2_NATIVE=0: the exact 4x Q8_0 repack)
        self.q2_native = os.environ.get("KT_GGUF_Q2_NATIVE", "1") == "1"
        if self.types[2] == GGML_Q2_0:
            self.type2 = GGML_Q2_0 if self.q2_native else GGML_Q8_0
        else:
            self.type2 = self.types[2]
        for t in (self.type13, self.type2):
            if t not in MMVQ_TYPES and not (t == GGML_Q2_0 and self.q2_native):
                raise RuntimeError(f"layer {kt_config.layer_idx}: ggml type {t} has no B200 kernel "
                                   f"(supported: {sorted(MMVQ_TYPES)})")
        self.moe_runner_config = None
        self._workspace = None

    def create_weights(self, layer, num_experts, hidden_size, intermediate_size_per_partition, params_dtype,
                       **extra_weight_attrs):
        E, N, K = num_experts, intermediate_size_per_partition, hidden_size
        self.N, self.K = N, K
        if N * self.world != self.reader.inter or K != self.reader.K:
            raise RuntimeError(f"GGUF experts {self.reader.inter}x{self.reader.K} vs layer {N}x{self.world} / {K}")
        if E == 0:
            return
        dev = torch.device("cuda", torch.cuda.current_device())
        w13 = Parameter(torch.empty((E, 2 * N, _row_bytes(K, self.type13)), dtype=torch.uint8, device=dev),
                        requires_grad=False)
        w2 = Parameter(torch.empty((E, K, _row_bytes(N, self.type2)), dtype=torch.uint8, device=dev), requires_grad=False)
        w13.weight_loader = w2.weight_loader = self._refuse_loader
        layer.register_parameter("w13_qweight", w13)
        layer.register_parameter("w2_qweight", w2)

    @staticmethod
    def _refuse_loader(param, loaded_weight, *a, **k):
        raise RuntimeError("GGUF hot experts take no checkpoint expert tensors")

    def process_weights_after_loading(self, layer) -> None:
        E = self.num_gpu_experts
        if E == 0:
            return
        try:
            from sglang.srt.eplb.expert_location_dispatch import get_global_expert_location_metadata

            meta = get_global_expert_location_metadata()
        except ImportError:
            meta = None
        p2l = meta.physical_to_logical_map_cpu[self.kt_config.layer_idx][:E].to(torch.int64) if meta is not None \
            else torch.arange(E)
        t0 = time.time()
        li, N = self.kt_config.layer_idx, self.N
        layer.w13_qweight.data[:, :N].copy_(self.reader.slice(li, "gate", N, self.rank, p2l))
        layer.w13_qweight.data[:, N:].copy_(self.reader.slice(li, "up", N, self.rank, p2l))
        down = self.reader.slice(li, "down", N, self.rank, p2l)
        if self.types[2] == GGML_Q2_0 and self.type2 == GGML_Q8_0:
            down = q2_0_to_q8_0(down)
        if tuple(down.shape) != tuple(layer.w2_qweight.shape):
            raise RuntimeError(f"down slice {tuple(down.shape)} vs slots {tuple(layer.w2_qweight.shape)}")
        layer.w2_qweight.data.copy_(down)
        if li == 0 or os.environ.get("KT_GGUF_HOT_LOG") == "1":
            mb = (layer.w13_qweight.numel() + layer.w2_qweight.numel()) / 1e6
            _log(f"rank {self.rank}: layer {li} {E} hot experts from the GGUF, types {self.types} -> "
                 f"({self.type13}, {self.type2}), {mb:.0f} MB on the GPU, {time.time() - t0:.1f} s")

    def create_moe_runner(self, layer, moe_runner_config):
        self.moe_runner_config = moe_runner_config

    def _use_prefill(self, x: torch.Tensor, T: int) -> bool:
        # layers of other types (a native Q2_0 down, the GEMV-only quantizations) run the GEMV at
        # every length, as the reference runs its window kernel for its Q2_0 layers
        return (PREFILL_ON_GPU and T >= PREFILL_MIN and x.dtype == torch.bfloat16 and self.K % 256 == 0
                and self.N % 256 == 0 and self.type13 in _multi.N.PREFILL_TYPES
                and self.type2 in _multi.N.PREFILL_TYPES)

    def apply(self, layer, dispatch_output):
        x = dispatch_output.hidden_states
        topk_weights, topk_ids, _ = dispatch_output.topk_output
        T, top_k = topk_ids.shape
        p13 = getattr(layer, "kt_kv_ptr13", None)  # KV-lent slots: per-slot pointer tables
        tbl = p13 is not None
        W13 = p13 if tbl else layer.w13_qweight
        W2 = layer.kt_kv_ptr2 if tbl else layer.w2_qweight
        ids = topk_ids.to(torch.int32)
        w = topk_weights.to(torch.float32)
        if self._use_prefill(x, T):
            n_slots = W13.numel() if tbl else W13.shape[0]
            need = _multi.N.load().kt_moe_prefill_workspace_size(T, top_k, self.K, self.N, n_slots)
            if self._workspace is None or self._workspace.numel() < need or self._workspace.device != x.device:
                self._workspace = _multi.N.workspace(need, x.device)
            out = _multi.moe_prefill(x, W13, W2, ids, w, self.type13, self.type2, self.N, table=tbl,
                                     workspace=self._workspace)
            return StandardCombineInput(hidden_states=out)
        # decode / verify windows and short extends: the reference's GEMV arithmetic
        h = _multi.moe_a8_vec_multi(x, W13, ids.reshape(-1), top_k, self.type13, 2 * self.N, T, tbl)
        h = _k.silu_and_mul(h)
        out = _multi.moe_a8_vec_multi(h, W2, ids.reshape(-1), 1, self.type2, self.K, T * top_k, tbl)
        return StandardCombineInput(hidden_states=_combine(out.view(T, top_k, self.K), w.view(T, top_k)))
