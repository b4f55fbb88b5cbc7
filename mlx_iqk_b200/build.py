"""Build step of the CUDA library: ``libiqk_b200.so`` for sm_100a, in-tree.

    python -m mlx_iqk_b200.build

nvcc cross-compiles without a GPU. The output sits beside this file, where
``kernels.library()`` loads it.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
SOURCES = ["iqk_capi.cu", "iqk_dense.cu", "iqk_dequant.cu", "iqk_ep.cu", "iqk_gemv.cu",
           "iqk_grouped.cu", "iqk_pack.cu", "iqk_static.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
         "--expt-relaxed-constexpr", "-diag-suppress", "177"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (Path(cand).exists() or cand == "nvcc"):
            return cand
    raise RuntimeError("nvcc not found")


def build(verbose: bool = False) -> Path:
    out = HERE / "libiqk_b200.so"
    srcs = [str(CSRC / s) for s in SOURCES]
    deps = (srcs + [str(p) for p in CSRC.glob("*.cuh")] + [str(p) for p in CSRC.glob("*.h")]
            + [str(HERE.parent / "include" / "iqk_b200.h")])
    if out.exists() and all(out.stat().st_mtime >= Path(d).stat().st_mtime for d in deps):
        return out
    tmp = out.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, *FLAGS, "-o", str(tmp), *srcs]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True, cwd=CSRC)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
