"""Hot GPU experts straight from a GGUF, for the KT hybrid — B200 (sm_100a) implementation.

Drop-in for sglang.srt.layers.moe.kt_gguf_hot (hot/kt_gguf_hot.py): KTGGUFHotExpertsMethod with
the reference's constructor, create_weights / process_weights_after_loading /
create_moe_runner / apply, the streams_hot_experts attribute, and the module helpers
BLOCK_INFO, MMVQ_TYPES, _row_bytes, q2_0_to_q8_0 and _combine. GPU slots 0..num_gpu_experts-1
hold this rank's tensor-parallel slice of each hot expert's raw GGUF blocks in the reference's
layout (hot/kt_gguf_hot.py:17-20):
  w13_qweight  uint8 [E_gpu, 2N, row_bytes(K, gate/up type)]   rows [gate; up]
  w2_qweight   uint8 [E_gpu, K,  row_bytes(N, down type)]
Routes with ids < 0 (experts on the CPU) contribute nothing.

GGUF access: GGUFExpertFile reads the expert tensors (blk.<l>.ffn_{gate,up,down}_exps.weight)
with gguf-py's memory-mapped reader, so loading a slot touches only that expert's pages.

apply() per MoE layer call:
- bf16 chunks of at least PREFILL_MIN tokens: the tcgen05 prefill layer
  (kt_gguf_moe_multi.moe_prefill: gate/up GEMM with SwiGLU, down GEMM, fp32 weighted sum), in
  place of the reference's streamed prefill (dequant to bf16 + CUTLASS fused MoE);
- smaller windows (decode, MTP verify, short extends): the q8_1 GEMV (moe_a8_vec_multi,
  bit-identical to the reference kernel), silu_and_mul, the GEMV on the down weights and the
  reference's combine (hot/kt_gguf_hot.py:240-304).
With KV-lent slots (layer.kt_kv_ptr13 / kt_kv_ptr2) both paths read the weights through the
per-slot pointer tables.

Types: the prefill layer takes Q8_0 (8), Q4_K (12), Q6_K (14) and IQ3_S (21); the GEMV also
Q4_0/Q4_1/Q5_0/Q5_1/IQ4_NL, Q2_K/Q3_K/Q5_K/IQ4_XS, IQ2_XXS/IQ2_XS/IQ2_S/IQ3_XXS/IQ1_S/IQ1_M and
the reference's Q2_0 (42); others raise at construction. As in the reference
(hot/kt_gguf_hot.py:21-25, 180-190) a Q2_0 down stays 2-bit on the GPU and its layer runs the
GEMV at every length; KT_GGUF_Q2_NATIVE=0 repacks it losslessly into Q8_0 (q2_0_to_q8_0),
which the prefill layer takes.
"""
import os
import time
from typing import Dict, Iterable, Tuple

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

# the decode combine is one kernel at every token count, bit-identical to out.mul_(w) + moe_sum
# (hot/kt_gguf_hot.py:37-38); the knob is read for compatibility
FUSED_COMBINE = os.environ.get("KT_HOT_FUSED_COMBINE", "1") == "1"
# bf16 chunks from this many tokens go through the tcgen05 prefill layer
PREFILL_MIN = int(os.environ.get("KT_B200_PREFILL_MIN", "128"))
PREFILL_ON_GPU = os.environ.get("KT_B200_PREFILL", "1") == "1"

GGML_Q8_0 = 8
GGML_Q2_0 = 42
# ggml type -> (values per block, bytes per block) for every type with a kernel here. IQ1_S is
# its 50-byte block (the reference's Python table says 74, IQ2_XS's size; its kernel's
# block_iq1_s is 50 bytes); IQ2_XS (17) and IQ1_M (29) are added.
BLOCK_INFO = {
    2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 20: (32, 18),
    10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210),
    16: (256, 66), 17: (256, 74), 18: (256, 98), 19: (256, 50), 21: (256, 110), 22: (256, 82), 23: (256, 136),
    29: (256, 56), 42: (64, 18),
}
# types a GPU slot may hold without a repack (Q2_0 only through q2_native)
MMVQ_TYPES = set(_multi.SUPPORTED_TYPES) - {GGML_Q2_0}


def _log(msg):
    print(f"[kt-gguf-hot {time.strftime('%H:%M:%S')}] {msg}", flush=True)


def _row_bytes(cols: int, t: int) -> int:
    """bytes of one row of `cols` values of ggml type t"""
    qk, nbytes = BLOCK_INFO[t]
    if cols % qk:
        raise ValueError(f"type {t} stores rows in blocks of {qk} values; {cols} is not a multiple")
    return cols // qk * nbytes


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


class GGUFExpertFile:
    """The MoE expert tensors of a GGUF file, read through gguf-py's memory map.

    E, inter and K come from the first layer's gate tensor (ggml shape [K, inter, E]); slices
    are copied out of the mapping, so only the pages of the requested experts are read."""

    PROJ = ("gate", "up", "down")

    def __init__(self, path: str):
        from gguf import GGUFReader

        self.path = path
        self._file = GGUFReader(path, "r")
        self._tensors = {t.name: t for t in self._file.tensors}
        self.layers = sorted({int(n.split(".")[1]) for n in self._tensors if n.endswith("ffn_gate_exps.weight")})
        if not self.layers:
            raise RuntimeError(f"{path}: no blk.<l>.ffn_gate_exps.weight tensors")
        ne = [int(v) for v in self._tensor(self.layers[0], "gate").shape]
        self.K, self.inter, self.E = ne[0], ne[1], ne[2]

    def _tensor(self, layer_idx: int, proj: str):
        name = f"blk.{layer_idx}.ffn_{proj}_exps.weight"
        t = self._tensors.get(name)
        if t is None:
            raise KeyError(f"{self.path}: no tensor {name}")
        return t

    def types(self, layer_idx: int) -> Tuple[int, int, int]:
        return tuple(int(self._tensor(layer_idx, p).tensor_type) for p in self.PROJ)

    def _bytes(self, layer_idx: int, proj: str) -> np.ndarray:
        """the tensor's raw bytes as [E, rows, row_bytes] (a view of the mapping)"""
        t = self._tensor(layer_idx, proj)
        rows = self.inter if proj != "down" else self.K
        return np.asarray(t.data).reshape(self.E, rows, -1)

    def slice(self, layer_idx: int, proj: str, N: int, rank: int, experts) -> torch.Tensor:
        """This rank's tensor-parallel part of the given experts, uint8 [len(experts), rows,
        bytes]: rows [N*rank, N*(rank+1)) of gate / up; of down, the block columns that hold
        the same N intermediate values."""
        e = np.asarray(experts, dtype=np.int64)
        raw = self._bytes(layer_idx, proj)
        if proj != "down":
            part = raw[e, N * rank:N * (rank + 1), :]
        else:
            qk, nbytes = BLOCK_INFO[int(self._tensor(layer_idx, "down").tensor_type)]
            if (N * rank) % qk or N % qk:
                raise ValueError(f"the down slice of {N} values at rank {rank} is not block aligned ({qk})")
            c0 = N * rank // qk * nbytes
            part = raw[e, :, c0:c0 + N // qk * nbytes]
        return torch.from_numpy(np.ascontiguousarray(part))


_readers: Dict[str, object] = {}


def _reader(path: str):
    """one reader per file, shared by every layer of the rank"""
    r = _readers.get(path)
    if r is None:
        r = _readers[path] = GGUFExpertFile(path)
    return r


def _slot_types(file_types: Tuple[int, int, int], q2_native: bool, layer_idx: int) -> Tuple[int, int]:
    """(gate/up type, down type) the GPU slots hold for a layer of these file types."""
    gate, up, down = file_types
    if gate != up:
        raise RuntimeError(f"layer {layer_idx}: the gate ({gate}) and up ({up}) tensors must share a GGUF type")
    slot_down = GGML_Q8_0 if down == GGML_Q2_0 and not q2_native else down
    for t in (gate, slot_down):
        if t not in MMVQ_TYPES and not (t == GGML_Q2_0 and q2_native):
            raise RuntimeError(f"layer {layer_idx}: GGUF type {t} has no B200 kernel "
                               f"(types with one: {sorted(MMVQ_TYPES | {GGML_Q2_0})})")
    return gate, slot_down


class KTGGUFHotExpertsMethod(FusedMoEMethodBase):
    """GPU-expert method the KT wrapper wraps when the experts are a GGUF."""

    # the reference skips this method at streamed-prefill sizes (its kernel is a decode kernel);
    # with the B200 prefill layer the method serves prefill chunks itself
    streams_hot_experts = not PREFILL_ON_GPU

    def __init__(self, kt_config, layer):
        self.kt_config = kt_config
        self.num_gpu_experts = kt_config.num_gpu_experts
        self.reader = _reader(kt_config.weight_path)
        self.rank, self.world = layer.moe_tp_rank, layer.moe_tp_size
        self.q2_native = os.environ.get("KT_GGUF_Q2_NATIVE", "1") == "1"
        self.types = tuple(self.reader.types(kt_config.layer_idx))
        self.type13, self.type2 = _slot_types(self.types, self.q2_native, kt_config.layer_idx)
        self.moe_runner_config = None
        self._workspace = None
        self.N = self.K = None

    def create_weights(self, layer, num_experts, hidden_size, intermediate_size_per_partition, params_dtype,
                       **extra_weight_attrs):
        self.N, self.K = intermediate_size_per_partition, hidden_size
        if (self.N * self.world, self.K) != (self.reader.inter, self.reader.K):
            raise RuntimeError(f"the GGUF's experts are {self.reader.inter} x {self.reader.K}; the layer asks for "
                               f"{self.N} x {self.world} ranks x {self.K}")
        if num_experts == 0:
            return
        dev = torch.device("cuda", torch.cuda.current_device())
        shapes = {"w13_qweight": (num_experts, 2 * self.N, _row_bytes(self.K, self.type13)),
                  "w2_qweight": (num_experts, self.K, _row_bytes(self.N, self.type2))}
        for name, shape in shapes.items():
            p = Parameter(torch.empty(shape, dtype=torch.uint8, device=dev), requires_grad=False)
            p.weight_loader = self._refuse_loader  # filled from the GGUF, never from a checkpoint
            layer.register_parameter(name, p)

    @staticmethod
    def _refuse_loader(param, loaded_weight, *a, **k):
        raise RuntimeError("the GGUF hot experts are read from the GGUF file, not loaded as checkpoint tensors")

    def _hot_experts(self, layer_idx: int) -> torch.Tensor:
        """logical expert of each GPU slot: the serving engine's placement map, else 0..E_gpu-1"""
        try:
            from sglang.srt.eplb.expert_location_dispatch import get_global_expert_location_metadata

            meta = get_global_expert_location_metadata()
        except ImportError:
            meta = None
        if meta is None:
            return torch.arange(self.num_gpu_experts)
        return meta.physical_to_logical_map_cpu[layer_idx][:self.num_gpu_experts].to(torch.int64)

    def slot_bytes(self, layer_idx: int, experts: Iterable[int]) -> Tuple[torch.Tensor, torch.Tensor]:
        """host bytes of the given experts in slot layout: (w13 [n, 2N, rb13], w2 [n, K, rb2])"""
        e = torch.as_tensor(list(experts) if not torch.is_tensor(experts) else experts, dtype=torch.int64)
        gate, up, down = (self.reader.slice(layer_idx, p, self.N, self.rank, e) for p in GGUFExpertFile.PROJ)
        if self.types[2] == GGML_Q2_0 and self.type2 == GGML_Q8_0:
            down = q2_0_to_q8_0(down)
        return torch.cat([gate, up], dim=1), down

    def process_weights_after_loading(self, layer) -> None:
        if self.num_gpu_experts == 0:
            return
        t0 = time.time()
        li = self.kt_config.layer_idx
        w13, w2 = self.slot_bytes(li, self._hot_experts(li))
        for param, src in ((layer.w13_qweight, w13), (layer.w2_qweight, w2)):
            if tuple(src.shape) != tuple(param.shape):
                raise RuntimeError(f"layer {li}: GGUF slice {tuple(src.shape)} does not fit the slots "
                                   f"{tuple(param.shape)}")
            param.data.copy_(src)
        if li == 0 or os.environ.get("KT_GGUF_HOT_LOG") == "1":
            mb = (layer.w13_qweight.numel() + layer.w2_qweight.numel()) / 1e6
            _log(f"rank {self.rank}: layer {li}: {self.num_gpu_experts} GPU experts ({mb:.0f} MB), GGUF types "
                 f"{self.types}, slots hold ({self.type13}, {self.type2}); {time.time() - t0:.1f} s")

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
        # the kernels take int32 ids and fp32 weights; no cast kernels when the router gave those
        ids = topk_ids if topk_ids.dtype == torch.int32 else topk_ids.to(torch.int32)
        w = topk_weights if topk_weights.dtype == torch.float32 else topk_weights.to(torch.float32)
        if self._use_prefill(x, T):
            n_slots = W13.numel() if tbl else W13.shape[0]
            need = _multi.N.load().kt_moe_prefill_workspace_size(T, top_k, self.K, self.N, n_slots)
            if self._workspace is None or self._workspace.numel() < need or self._workspace.device != x.device:
                self._workspace = _multi.N.workspace(need, x.device)
            out = _multi.moe_prefill(x, W13, W2, ids, w, self.type13, self.type2, self.N, table=tbl,
                                     workspace=self._workspace)
            return StandardCombineInput(hidden_states=out)
        # decode / verify windows and short extends: the reference's GEMV arithmetic
        flat = ids.reshape(-1)
        h = _multi.moe_a8_vec_multi(x, W13, flat, top_k, self.type13, 2 * self.N, T, tbl)
        h = _k.silu_and_mul(h)
        out = _multi.moe_a8_vec_multi(h, W2, flat, 1, self.type2, self.K, T * top_k, tbl)
        return StandardCombineInput(hidden_states=_combine(out.view(T, top_k, self.K), w.reshape(T, top_k)))
