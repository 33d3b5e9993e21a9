"""GGUF formats and the CPU oracle's dequantizers against the golden vectors (no GPU).

The library's code books are pinned to the reference's tables (hot/kt_gguf_moe_multi/
ggml-common.h) through committed SHA-256 digests (tests/golden/make_reference_digests.py);
with KT_REFERENCE_ROOT set to a reference checkout the tables are also compared directly."""
import hashlib
import json
import os
import re
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = np.load(Path(__file__).with_name("golden") / "gguf_dequant.npz")
TYPES = (8, 12, 14, 21)
# the GEMV's wider type switch: 32-value blocks and the K-quants Q2_K / Q3_K / Q5_K / IQ4_XS
LEGACY = (2, 3, 6, 7, 20, 10, 11, 13, 23, 42, 16, 17, 18, 19, 22, 29)  # Q2_0 and the code-book i-quants too
DIGESTS = json.loads((Path(__file__).with_name("golden") / "reference_table_digests.json").read_text())
_REF_ROOT = os.environ.get("KT_REFERENCE_ROOT")
REF_COMMON = Path(_REF_ROOT) / "hot" / "kt_gguf_moe_multi" / "ggml-common.h" if _REF_ROOT else None
needs_reference = pytest.mark.skipif(REF_COMMON is None or not REF_COMMON.exists(),
                                     reason="KT_REFERENCE_ROOT does not name a reference checkout")


def _digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).astype(a.dtype.newbyteorder("<")).tobytes()).hexdigest()


def test_block_sizes_known_answers():
    # hot/kt_gguf_hot.py:76-80 BLOCK_INFO for the hot-path types
    assert O.BLOCK == {8: (32, 34), 12: (256, 144), 14: (256, 210), 21: (256, 110),
                       2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 20: (32, 18),
                       10: (256, 84), 11: (256, 110), 13: (256, 176), 23: (256, 136), 42: (64, 18),
                       16: (256, 66), 17: (256, 74), 18: (256, 98), 19: (256, 50), 22: (256, 82), 29: (256, 56)}
    from kt_gguf_b200 import synth

    assert synth.BLOCK == O.BLOCK
    assert O.row_bytes(12, 2048) == 8 * 144 and O.row_bytes(14, 512) == 420 and O.row_bytes(21, 512) == 220


@pytest.mark.parametrize("qtype", TYPES + LEGACY)
def test_oracle_dequant_matches_golden_bit_exact(qtype):
    blocks = GOLDEN[f"{qtype}_blocks"]
    want = GOLDEN[f"{qtype}_values"]
    got = O.dequant(qtype, blocks, 512)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_iq3s_grid_matches_golden_and_header():
    import importlib.util

    from kt_gguf_b200 import synth  # noqa: F401  (package importable)

    header = Path(__file__).resolve().parents[1] / "kt-prefill-lend_b200" / "csrc" / "iq3s_grid.h"
    words = [int(x, 16) for x in re.findall(r"0x([0-9a-f]{8})u", header.read_text())]
    assert np.array_equal(np.array(words, dtype=np.uint32), GOLDEN["iq3s_grid"])
    assert importlib.util.find_spec("gguf") is not None


def test_code_books_match_reference_digests():
    # the device code books in the form the reference's tables hold them: iq3s / iq3xxs as uint32,
    # iq2xxs / iq2xs / iq2s as uint64 (byte j = element j), iq1s_grid_gpu in its nibble form
    words = {"iq3s_grid": GOLDEN["iq3s_grid"].astype(np.uint32), "iq3xxs_grid": _header_words("IQ3XXS")}
    for name, key in (("iq2xxs_grid", "IQ2XXS"), ("iq2xs_grid", "IQ2XS"), ("iq2s_grid", "IQ2S")):
        words[name] = _header_words(key).view(np.uint64)
    words["iq1s_grid_gpu"] = _header_words("IQ1S").astype(np.uint64)
    for name, arr in words.items():
        want = DIGESTS[name]
        assert arr.dtype.name == want["dtype"] and arr.size == want["count"], name
        assert _digest(arr) == want["sha256"], name


@needs_reference
def test_iq3s_grid_matches_reference_table():
    # the reference's own codebook (ggml-common.h:598-665), read as text
    src = REF_COMMON.read_text()
    body = re.search(r"iq3s_grid\[512\]\s*=\s*\{(.*?)\};", src, re.S).group(1)
    ref = np.array([int(x, 16) for x in re.findall(r"0x[0-9a-fA-F]+", body)], dtype=np.uint32)
    assert np.array_equal(ref, GOLDEN["iq3s_grid"])


def _header_words(name):
    header = Path(__file__).resolve().parents[1] / "kt-prefill-lend_b200" / "csrc" / "iquant_grids.h"
    body = re.search(r"#define KT_" + name + r"_GRID_INIT \{(.*?)\}", header.read_text(), re.S).group(1)
    return np.array([int(x, 16) for x in re.findall(r"0x([0-9a-f]{8})u", body)], dtype=np.uint32)


def test_iquant_books_match_gguf_py():
    # iquant_grids.h as committed against gguf-py's code books (the generator's source)
    from gguf.quants import IQ1_S, IQ2_S, IQ2_XS, IQ2_XXS, IQ3_XXS

    def entries(cls):
        cls.init_grid()
        return cls.grid.reshape(cls.grid_shape).astype(np.int64)

    for name, cls in (("IQ2XXS", IQ2_XXS), ("IQ2XS", IQ2_XS), ("IQ2S", IQ2_S), ("IQ3XXS", IQ3_XXS)):
        w = _header_words(name)
        got = np.stack([(w >> (8 * k)) & 0xff for k in range(4)], axis=-1).reshape(entries(cls).shape)
        assert np.array_equal(got, entries(cls)), name
    w = _header_words("IQ1S")
    nib = np.stack([(w >> (8 * k + 4 * h)) & 0xf for h in range(2) for k in range(4)], axis=-1).astype(np.int64) - 1
    assert np.array_equal(nib, entries(IQ1_S))
    # the sign table the kernels compute: 7 bits + even parity
    ks = np.frombuffer(IQ2_XXS.ksigns, dtype=np.uint8)
    assert all(int(ks[i]) == i | ((bin(i).count("1") & 1) << 7) for i in range(128))


@needs_reference
def test_iquant_books_match_reference_tables():
    # the reference's ggml-common.h tables (read as text): iq2xxs_grid, iq2xs_grid, iq2s_grid
    # (uint64, byte j = element j), iq3xxs_grid, and iq1s_grid_gpu (the nibble form)
    src = REF_COMMON.read_text()

    def ref(name, dt):
        body = re.search(name + r"\[\d+\]\s*=\s*\{(.*?)\};", src, re.S).group(1)
        return np.array([int(x, 16) for x in re.findall(r"0x[0-9a-fA-F]+", body)], dtype=dt)

    assert np.array_equal(ref("iq2xxs_grid", np.uint64).view(np.uint32), _header_words("IQ2XXS"))
    assert np.array_equal(ref("iq2xs_grid", np.uint64).view(np.uint32), _header_words("IQ2XS"))
    assert np.array_equal(ref("iq2s_grid", np.uint64).view(np.uint32), _header_words("IQ2S"))
    assert np.array_equal(ref("iq3xxs_grid", np.uint32), _header_words("IQ3XXS"))
    assert np.array_equal(ref("iq1s_grid_gpu", np.uint64).astype(np.uint32), _header_words("IQ1S"))


@pytest.mark.parametrize("qtype,tol", [(8, 0.01), (12, 0.12), (14, 0.03), (21, 0.25)])
def test_encoder_round_trip(qtype, tol):
    from kt_gguf_b200 import synth

    rng = np.random.default_rng(qtype)
    x = rng.standard_normal((16, 1024), dtype=np.float32) * 0.02
    back = O.dequant(qtype, synth.quantize(x, qtype), 1024)
    assert O.rel_l2(back, x) < tol


def test_q8_1_known_answers():
    # d = amax/127, q = roundf(x/d), s = sum of the unquantized values, zero padding to 512
    x = np.zeros((1, 40), dtype=np.float32)
    x[0, :32] = np.arange(32) - 16.0  # amax 16
    x[0, 32:40] = 0.5
    q = O.quantize_q8_1(x)
    assert q.shape == (1, 16 * 36)
    d = q[0, 0:2].view(np.float16)[0]
    s = q[0, 2:4].view(np.float16)[0]
    assert d == np.float16(16 / 127) and s == np.float16(-16.0)
    codes = q[0, 4:36].view(np.int8)
    assert np.array_equal(codes, np.round((np.arange(32) - 16) * 127 / 16).astype(np.int8))
    blk1 = q[0, 36:72]
    assert blk1[0:2].view(np.float16)[0] == np.float16(0.5 / 127)
    assert np.all(blk1[4:12].view(np.int8) == 127) and np.all(blk1[12:36] == 0)
    assert np.all(q[0, 72:] == 0)  # all-zero padded blocks: d = 0, s = 0, q = 0


def test_bf16_helpers_round_to_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.0e38, 1e-40, np.inf], dtype=np.float32)
    b = O.f32_to_bf16(x)
    back = O.bf16_to_f32(b)
    import torch

    want = torch.from_numpy(x).to(torch.bfloat16).to(torch.float32).numpy()
    assert np.array_equal(back.view(np.uint32), want.view(np.uint32))


def test_iq4nl_levels_match_gguf_py_and_device_words():
    # the code book the device packs into four words (gguf_dot.cuh KT_IQ4NL_W0..3)
    levels = GOLDEN["iq4nl_levels"].astype(np.int8)
    src = (Path(__file__).resolve().parents[1] / "kt-prefill-lend_b200" / "csrc" / "gguf_dot.cuh").read_text()
    words = [int(re.search(rf"#define KT_IQ4NL_W{i} (0x[0-9A-Fa-f]+)u", src).group(1), 16) for i in range(4)]
    packed = np.array(words, dtype=np.uint32).view(np.int8)
    assert np.array_equal(packed, levels)
