"""Build recipe for the reference's own sparse-conv CUDA kernels, a test-only checker.

Compiles ``oracle/ref_libsparse.cpp`` (our binding) with the reference's unmodified
``BK/ops/libsparse/conv.cu``, read where it lies in the reference checkout, for sm_100a
into ``oracle/_ref/vdit_ref_libsparse.so`` (git-ignored; it is copied to GPU machines with
the other built libraries).  The checkout is an argument, else ``VDIT_REFERENCE_DIR``;
without either the build is skipped.  The reference's own
build system (its setup.py, which also pulls in its attention and mesh sources) is not
used.

    python oracle/build_ref.py <reference-root>
"""
from __future__ import annotations

import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CONV_IN_CHECKOUT = Path("baseline_repo/3dgen-main/ops/libsparse/conv.cu")
OUT_DIR = HERE / "_ref"
OUT = OUT_DIR / "vdit_ref_libsparse.so"
NAME = "vdit_ref_libsparse"


def build(ref_root=None, verbose: bool = False):
    """Returns the built library's path, or None without the reference checkout."""
    if ref_root is None:
        from oracle import reference_root
        ref_root = reference_root()
    if ref_root is None or not (Path(ref_root) / CONV_IN_CHECKOUT).exists():
        return None
    sources = [HERE / "ref_libsparse.cpp", Path(ref_root) / CONV_IN_CHECKOUT]
    if OUT.exists() and OUT.stat().st_mtime >= max(s.stat().st_mtime for s in sources):
        return OUT
    bdir = OUT_DIR / "build"
    bdir.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils.cpp_extension import load
    load(name=NAME, sources=[str(s) for s in sources], build_directory=str(bdir),
         extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"],
         verbose=verbose, is_python_module=True)
    shutil.copy2(bdir / f"{NAME}.so", OUT)
    return OUT


def load_built():
    """Import the prebuilt checker module (None when it was not built)."""
    if not OUT.exists():
        return None
    import importlib.machinery
    import importlib.util
    import torch  # noqa: F401  (the module links against torch's libraries)
    loader = importlib.machinery.ExtensionFileLoader(NAME, str(OUT))
    spec = importlib.util.spec_from_loader(NAME, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    sys.path.insert(0, str(HERE.parent))
    print(build(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True))
