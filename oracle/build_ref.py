"""Builds the reference's GGUF MoE GEMV kernel into oracle/_ref/ — TEST INFRASTRUCTURE ONLY.

Compiles hot/kt_gguf_moe_multi/kt_gguf_moe_multi.cu from the mounted reference tree (read in
place, never copied) with oracle/ref_binding.cpp, for sm_100a, with the macro settings of the
reference's loader (hot/kt_gguf_moe_multi.py:55-74): the window build (KT_MAXM=4,
KT_MMV_Y=2, KT_RPW=4) and the per-route build (KT_PER_ROUTE=1). The resulting Python
modules travel to the GPU box with the tree; load() imports them there without the
reference sources. Nothing in the product imports them.

Usage: KT_REFERENCE_ROOT=<reference checkout> python oracle/build_ref.py
"""
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
# the reference checkout is named by KT_REFERENCE_ROOT; without it nothing is built
_ROOT = os.environ.get("KT_REFERENCE_ROOT")
REF_DIR = Path(_ROOT) / "hot" / "kt_gguf_moe_multi" if _ROOT else None
VARIANTS = {
    "kt_ref_window": ["-DKT_MAXM=4", "-DKT_MMV_Y=2", "-DKT_RPW=4", "-DKT_PER_ROUTE=0", "-DKT_PTR_TABLE=0"],
    "kt_ref_routes": ["-DKT_MAXM=4", "-DKT_MMV_Y=2", "-DKT_RPW=4", "-DKT_PER_ROUTE=1", "-DKT_PTR_TABLE=0"],
}


def _so(name: str) -> Path:
    return OUT / name / f"{name}.so"


def build(variants=None) -> None:
    if REF_DIR is None or not REF_DIR.exists():
        return
    names = [n for n in (variants or VARIANTS) if not _so(n).exists()]
    if not names:
        return
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from concurrent.futures import ThreadPoolExecutor

    from torch.utils.cpp_extension import load

    def one(name):
        d = OUT / name
        d.mkdir(parents=True, exist_ok=True)
        load(name=name, sources=[str(HERE / "ref_binding.cpp"), str(REF_DIR / "kt_gguf_moe_multi.cu")],
             extra_cuda_cflags=["-O3", f"-I{REF_DIR}", *VARIANTS[name]], extra_include_paths=[str(REF_DIR)],
             build_directory=str(d), verbose=False)

    with ThreadPoolExecutor(len(names)) as ex:
        list(ex.map(one, names))


def available(name: str) -> bool:
    return _so(name).exists()


def load_module(name: str):
    """Imports a built reference module (torch must be importable)."""
    import torch  # noqa: F401  (the module links against torch)

    spec = importlib.util.spec_from_file_location(name, _so(name))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    build()
    print({n: available(n) for n in VARIANTS})
    sys.exit(0)
