"""Generates tests/golden/gguf_dequant.npz: known-answer vectors for the GGUF dequantizers.

The reference ships no fixtures for this path, so the known answers come from gguf-py
0.19.0 (`gguf.quants.dequantize`, numpy restatements of ggml's dequantize_row_*), an
implementation independent of this repository. For each type the file holds
  <type>_blocks  uint8  : 48 rows of 512 values (2 super-blocks / 16 32-value blocks per row):
                           rows 0-23 encoded from N(0, 0.02) weights (gguf_encode.c for the
                           hot-path types, gguf-py's quantizer for Q4_0/Q4_1/Q5_0/Q5_1; IQ4_NL,
                           which neither encodes, takes random blocks here too),
                           rows 24-47 random bytes with finite scales (every code pattern)
  <type>_values  float32: gguf-py's dequantization of those rows
and for Q2_K, Q3_K, Q5_K, IQ4_XS and the code-book i-quants IQ2_XXS, IQ2_XS, IQ2_S, IQ3_XXS,
IQ1_S, IQ1_M, which gguf-py does not encode, 48 rows of random blocks with finite scales and
their dequantization; for the reference's own Q2_0 (ggml type 42,
unknown to gguf-py) 24 encoded and 24 random rows with values (code - 1) * d computed here
in numpy from the block's definition (kt_gguf_moe_multi.cu:33-46 of the reference),
plus the IQ3_S codebook as uint32 words and the IQ4_NL levels.

Run from the repository root: python tests/golden/make_golden.py
"""
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "kt-prefill-lend_b200"))

from gguf import GGMLQuantizationType as Q  # noqa: E402
from gguf.quants import IQ3_S, IQ4_NL, dequantize, quantize  # noqa: E402

from kt_gguf_b200 import synth  # noqa: E402

TYPES = {8: Q.Q8_0, 12: Q.Q4_K, 14: Q.Q6_K, 21: Q.IQ3_S}
LEGACY = {2: Q.Q4_0, 3: Q.Q4_1, 6: Q.Q5_0, 7: Q.Q5_1, 20: Q.IQ4_NL}
KQUANTS = {10: Q.Q2_K, 11: Q.Q3_K, 13: Q.Q5_K, 23: Q.IQ4_XS}
IQUANTS = {16: Q.IQ2_XXS, 17: Q.IQ2_XS, 18: Q.IQ3_XXS, 19: Q.IQ1_S, 22: Q.IQ2_S, 29: Q.IQ1_M}


def main():
    rng = np.random.default_rng(20261201)
    out = {}
    for t, qt in TYPES.items():
        enc = synth.quantize(rng.standard_normal((24, 512), dtype=np.float32) * 0.02, t)
        rnd = synth.random_blocks(rng, t, 24, 512)
        blocks = np.concatenate([enc, rnd])
        out[f"{t}_blocks"] = blocks
        out[f"{t}_values"] = dequantize(blocks, qt).reshape(48, 512).astype(np.float32)
    for t, qt in LEGACY.items():
        w = rng.standard_normal((24, 512), dtype=np.float32) * 0.02
        enc = synth.random_blocks(rng, t, 24, 512) if t == 20 else quantize(w, qt)
        rnd = synth.random_blocks(rng, t, 24, 512)
        blocks = np.concatenate([enc, rnd])
        out[f"{t}_blocks"] = blocks
        out[f"{t}_values"] = dequantize(blocks, qt).reshape(48, 512).astype(np.float32)
    for t, qt in KQUANTS.items():
        blocks = synth.random_blocks(rng, t, 48, 512)
        out[f"{t}_blocks"] = blocks
        out[f"{t}_values"] = dequantize(blocks, qt).reshape(48, 512).astype(np.float32)
    enc = synth.quantize(rng.standard_normal((24, 512), dtype=np.float32) * 0.02, 42)
    blocks = np.concatenate([enc, synth.random_blocks(rng, 42, 24, 512)])
    b = blocks.reshape(48, 8, 18)
    d = b[:, :, :2].copy().view(np.float16).astype(np.float32)  # [48, 8, 1]
    codes = ((b[:, :, 2:, None] >> np.array([0, 2, 4, 6], dtype=np.uint8)) & 3).reshape(48, 8, 64)
    out["42_blocks"] = blocks
    out["42_values"] = ((codes.astype(np.float32) - 1) * d).reshape(48, 512)
    for t, qt in IQUANTS.items():
        blocks = synth.random_blocks(rng, t, 48, 512)
        out[f"{t}_blocks"] = blocks
        out[f"{t}_values"] = dequantize(blocks, qt).reshape(48, 512).astype(np.float32)
    out["iq4nl_levels"] = np.array(IQ4_NL.kvalues, dtype=np.int8)
    IQ3_S.init_grid()
    g = IQ3_S.grid.reshape(512, 4).astype(np.uint32)
    out["iq3s_grid"] = g[:, 0] | (g[:, 1] << 8) | (g[:, 2] << 16) | (g[:, 3] << 24)
    path = Path(__file__).with_name("gguf_dequant.npz")
    np.savez_compressed(path, **out)
    print(path, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
