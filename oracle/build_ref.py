"""Build the reference's own CUDA op (cashcon57/open-supersampling
oss/cuda/src: bindings.cpp, rasterizer_fwd.cu, rasterizer_bwd.cu,
tile_bin_counting_sort.cu, compiled where they lie, unmodified) for sm_100a
into oracle/_ref/_C.so.

TEST INFRASTRUCTURE ONLY: the result is the kernel-level speed bar bench.py
times beside the product and a coarse cross-check; nothing on the product path
imports it.  The reference's own setup.py targets sm_80-sm_90 only; this recipe
compiles the same four sources with the same nvcc flags plus an sm_100a
gencode through torch.utils.cpp_extension.

    python oracle/build_ref.py [--reference /path/to/open-supersampling]

Needs the reference tree (present where the build runs); the built .so is
what travels to a GPU box.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
OUT_DIR = ORACLE_DIR / "_ref"
SOURCES = ("bindings.cpp", "rasterizer_fwd.cu", "rasterizer_bwd.cu", "tile_bin_counting_sort.cu")
# the reference setup.py's nvcc flags (oss/cuda/setup.py:6-18) with the gencode list replaced
NVCC_FLAGS = ["-O3", "-std=c++17", "--expt-relaxed-constexpr", "--expt-extended-lambda", "-ftz=true",
              "-prec-div=false", "-lineinfo", "-gencode=arch=compute_100a,code=sm_100a"]


def built() -> Path | None:
    so = OUT_DIR / "_C.so"
    return so if so.exists() else None


def up_to_date(reference: Path) -> bool:
    so = built()
    if so is None:
        return False
    src = reference / "oss" / "cuda" / "src"
    inputs = [src / s for s in SOURCES] + [src / "common.cuh", Path(__file__)]
    return all(so.stat().st_mtime >= p.stat().st_mtime for p in inputs if p.exists())


def build(reference: Path) -> Path:
    """Compile the four reference sources in place into oracle/_ref/_C.so
    (incremental: ninja rebuilds only what changed)."""
    src = reference / "oss" / "cuda" / "src"
    missing = [s for s in SOURCES if not (src / s).exists()]
    if missing:
        raise FileNotFoundError(f"reference sources not found under {src}: {missing}")
    if up_to_date(reference):
        return OUT_DIR / "_C.so"
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    from torch.utils.cpp_extension import load

    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    load(name="_C", sources=[str(src / s) for s in SOURCES], extra_cflags=["-O3", "-std=c++17"],
         extra_cuda_cflags=NVCC_FLAGS, build_directory=str(OUT_DIR), verbose=False)
    return OUT_DIR / "_C.so"


def load_built():
    """Import oracle/_ref/_C.so (raises ImportError if it was not built)."""
    import importlib.util

    so = built()
    if so is None:
        raise ImportError("oracle/_ref/_C.so not built (python oracle/build_ref.py)")
    import torch  # noqa: F401 - the extension links against libtorch

    # the binding's PyInit symbol fixes the module name to _C; it is registered
    # under a distinct key so it never shadows the product's oss_cuda._C
    spec = importlib.util.spec_from_file_location("_C", so)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("OSS_REFERENCE_DIR"),
                    help="the reference checkout (default: $OSS_REFERENCE_DIR)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or OSS_REFERENCE_DIR")
    print(build(Path(args.reference)))
    sys.exit(0)
