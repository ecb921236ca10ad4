"""Builds libesm_b200.so in-tree for sm_100a with nvcc (no JIT, no torch extension machinery).

    python codon-infer_b200/build.py [--force]

Objects go to codon-infer_b200/_build/, the library to codon-infer_b200/libesm_b200.so.
The CUDA runtime is linked statically; the driver API is reached through
cudaGetDriverEntryPoint, so the library loads (and its host-only entry points run) on machines
without a GPU.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libesm_b200.so"
INCLUDE = PKG.parent / "include"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3,-ffp-contract=off", "-I", str(INCLUDE)]
SOURCES = ["gemm_tc.cu", "kernels.cu", "attention.cu", "attention_tc3.cu", "contact_tc.cu", "quantize.cu", "contact_rank.cu", "esm_api.cu", "esm_group.cpp", "formats.cpp", "noalloc.cu"]


def _needs(obj: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    jobs = []
    objs = []
    for src in SOURCES:
        s = CSRC / src
        o = BUILD / (src.rsplit(".", 1)[0] + ".o")
        objs.append(o)
        if force or _needs(o, [s] + headers):
            lang = ["-x", "cu"] if src.endswith(".cu") else ["-x", "c++"]
            jobs.append([NVCC, *ARCH, *COMMON, *lang, "-c", str(s), "-o", str(o)])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        list(ex.map(run, jobs))
    if force or jobs or _needs(LIB, objs):
        run([NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lpthread", "-ldl", "-lrt"])
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
