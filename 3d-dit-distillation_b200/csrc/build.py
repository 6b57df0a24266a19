"""Build ``libvdit.so`` (sm_100a) in-tree with nvcc.

Each ``.cu`` file compiles to an object under ``_build/`` (rebuilt only when
it or a header is newer), then the objects link into
``3d-dit-distillation_b200/libvdit.so`` with a static CUDA runtime, so the
library loads on a machine without a GPU or a matching libcudart.

    python 3d-dit-distillation_b200/csrc/build.py [--verbose] [--ptxas-info]
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
ROOT = PKG.parent
OUT = PKG / "libvdit.so"
BUILD = ROOT / "_build"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-I", str(ROOT / "include")]


# per-file extra flags: the attention kernel keeps a 128-column score row in
# registers per thread (224 threads, one CTA per SM), so it may use up to 200.
EXTRA = {"attention.cu": ["-maxrregcount=200"]}


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _compile(src: Path, ptxas_info: bool, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if obj.exists() and obj.stat().st_mtime >= newest_dep and not ptxas_info:
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, *EXTRA.get(src.name, []), "-c", str(src), "-o", str(obj)]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if ptxas_info or verbose:
        sys.stdout.write(r.stderr)
    return obj


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, ptxas_info, verbose), srcs))
    if OUT.exists() and OUT.stat().st_mtime >= max(o.stat().st_mtime for o in objs):
        return OUT
    cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(OUT), *map(str, objs),
           "-Xlinker", "--no-undefined", "-ldl", "-lrt", "-lpthread"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, ptxas_info="--ptxas-info" in sys.argv))
