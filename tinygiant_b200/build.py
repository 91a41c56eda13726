"""Build libtinygiant.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python -m tinygiant_b200.build [-v] [--incremental]

The library lands next to this file (tinygiant_b200/libtinygiant.so), where
tinygiant_b200/_lib.py finds it, as the reference's _lib.find_library does.
By default every object is rebuilt from its source (stale objects copied in
from elsewhere can never be linked); --incremental rebuilds only objects older
than their sources or headers.  Sources compile in parallel.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT = PKG / "libtinygiant.so"
SOURCES = ["tg_kernels.cu", "tg_decode.cu", "tg_batched.cu", "tg_tc.cu", "tg_kquant.cu", "tg_capi.cu", "tg_ep.cu",
           "tg_noalloc.cu", "tg_attn.cu"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (Path(c).exists() or c == "nvcc"):
            return c
    return "nvcc"


def sources() -> list[Path]:
    return [CSRC / s for s in SOURCES if (CSRC / s).exists()]


def clean() -> None:
    """Remove the library and every object of this package."""
    for p in [OUT, *CSRC.glob("*.o")]:
        if p.exists():
            p.unlink()


def build(verbose: bool = False, extra: list[str] | None = None, incremental: bool = False) -> Path:
    if not incremental:
        clean()
    srcs = sources()
    hdrs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [PKG.parent / "include" / "tinygiant.h"]

    def stale(src: Path, obj: Path) -> bool:
        return not obj.exists() or any(d.stat().st_mtime > obj.stat().st_mtime for d in [src, *hdrs] if d.exists())

    def compile_one(src: Path) -> Path:
        obj = CSRC / (src.stem + ".o")
        if stale(src, obj):
            cmd = [nvcc(), *NVCC_FLAGS, *(extra or []), "-c", str(src), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
        return obj

    with ThreadPoolExecutor(max_workers=max(1, min(len(srcs), os.cpu_count() or 1))) as ex:
        objs = list(ex.map(compile_one, srcs))
    if not OUT.exists() or any(o.stat().st_mtime > OUT.stat().st_mtime for o in objs):
        cmd = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *map(str, objs), "-o", str(OUT)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, incremental="--incremental" in sys.argv))
