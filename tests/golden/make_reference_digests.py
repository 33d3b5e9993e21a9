"""Writes tests/golden/reference_table_digests.json: SHA-256 digests of the code books in the
reference's ggml-common.h (hot/kt_gguf_moe_multi/ggml-common.h:598-665 for iq3s_grid, and the
iq2xxs / iq2xs / iq2s / iq3xxs / iq1s_grid_gpu tables), parsed as text into little-endian
arrays of the table's element type. The CPU tests compare the library's code books against
these digests, so the pin holds where the reference tree is absent.

Usage: KT_REFERENCE_ROOT=<reference checkout> python tests/golden/make_reference_digests.py
"""
import hashlib
import json
import os
import re
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).with_name("reference_table_digests.json")
# table name in ggml-common.h -> element type
TABLES = {"iq3s_grid": np.uint32, "iq2xxs_grid": np.uint64, "iq2xs_grid": np.uint64, "iq2s_grid": np.uint64,
          "iq3xxs_grid": np.uint32, "iq1s_grid_gpu": np.uint64}


def parse(src: str, name: str, dtype) -> np.ndarray:
    body = re.search(name + r"\[\d+\]\s*=\s*\{(.*?)\};", src, re.S).group(1)
    return np.array([int(x, 16) for x in re.findall(r"0x[0-9a-fA-F]+", body)], dtype=dtype)


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).astype(a.dtype.newbyteorder("<")).tobytes()).hexdigest()


def main() -> int:
    root = os.environ.get("KT_REFERENCE_ROOT")
    if not root:
        print("set KT_REFERENCE_ROOT to the reference checkout", file=sys.stderr)
        return 1
    src = (Path(root) / "hot" / "kt_gguf_moe_multi" / "ggml-common.h").read_text()
    out = {name: {"dtype": np.dtype(dt).name, "count": int(parse(src, name, dt).size),
                  "sha256": digest(parse(src, name, dt))} for name, dt in TABLES.items()}
    OUT.write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print(OUT)
    return 0


if __name__ == "__main__":
    sys.exit(main())
