"""The hot method's GGUF access (kt_gguf_hot.GGUFExpertFile) on a real GGUF file written with
gguf-py: expert counts and sizes from the tensor shapes, ggml types, and the tensor-parallel
slices of gate / up rows and down block columns the GPU slots are filled from (no GPU)."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from kt_gguf_b200 import kt_gguf_hot as H

from gguf_fixture import E, INTER, K, write_gguf


def test_gguf_expert_file_geometry_and_tp_slices(tmp_path):
    path = tmp_path / "experts.gguf"
    data = write_gguf(path)
    f = H.GGUFExpertFile(str(path))
    assert (f.E, f.inter, f.K, f.layers) == (E, INTER, K, [0, 1])
    assert f.types(1) == (12, 12, 14)
    experts = torch.tensor([4, 1, 5])
    for rank in (0, 1):  # two tensor-parallel ranks of 256 intermediate rows each
        N = INTER // 2
        for proj in ("gate", "up"):
            got = f.slice(1, proj, N, rank, experts)
            assert torch.equal(got, torch.from_numpy(data[(1, proj)][[4, 1, 5], N * rank:N * (rank + 1)]))
        down = f.slice(1, "down", N, rank, experts)  # Q6_K: 210 bytes per 256 values
        assert torch.equal(down, torch.from_numpy(data[(1, "down")][[4, 1, 5], :, 210 * rank:210 * (rank + 1)]))
    with pytest.raises(ValueError):
        f.slice(0, "down", 100, 1, experts)  # not block aligned
    with pytest.raises(KeyError):
        f.types(7)


def test_method_slot_bytes_from_the_file(tmp_path):
    path = tmp_path / "experts.gguf"
    data = write_gguf(path, seed=2)
    H._readers.pop(str(path), None)
    kt = SimpleNamespace(num_gpu_experts=3, weight_path=str(path), layer_idx=0)
    m = H.KTGGUFHotExpertsMethod(kt, SimpleNamespace(moe_tp_rank=0, moe_tp_size=1))
    assert (m.type13, m.type2) == (12, 14) and m.reader is H._reader(str(path))
    m.N, m.K = INTER, K
    w13, w2 = m.slot_bytes(0, [2, 0])
    assert torch.equal(w13[:, :INTER], torch.from_numpy(data[(0, "gate")][[2, 0]]))
    assert torch.equal(w13[:, INTER:], torch.from_numpy(data[(0, "up")][[2, 0]]))
    assert torch.equal(w2, torch.from_numpy(data[(0, "down")][[2, 0]]))


def test_method_rejects_mixed_gate_up_types(tmp_path):
    path = tmp_path / "mixed.gguf"
    write_gguf(path, types=(12, 14, 14))
    kt = SimpleNamespace(num_gpu_experts=3, weight_path=str(path), layer_idx=0)
    with pytest.raises(RuntimeError, match="share"):
        H.KTGGUFHotExpertsMethod(kt, SimpleNamespace(moe_tp_rank=0, moe_tp_size=1))
