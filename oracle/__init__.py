"""CPU oracle for the sparse-voxel DiT (lat_dit) forward path.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this
directory; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg may import it, and only as the checker or the timed CPU
baseline.  The product path fails loudly when its CUDA library is missing.

Contents
--------
``geometry``  numpy restatement of the per-sample static geometry
              (lexicographic permutation, 16-level Hilbert codes for the four
              window orders, window ``cu_seqlens``, 27-neighbour
              ``conv_indices``, 3D/2D RoPE tables).  Integer results are
              bit-exact with the reference.
``model``     torch-fp32 CPU restatement of ``FlowModel.forward`` (cond and
              zero-context uncond), the exact 1-token uncond branch, the
              depthwise and dense 27-tap sparse convolutions and the exact
              Euler+CFG sampler.

Parity of both modules is pinned against fixtures produced by running the
reference itself on CPU (``tests/golden/make_golden.py``).
"""

import os as _os
from pathlib import Path as _Path


def reference_root():
    """The reference checkout named by the ``VDIT_REFERENCE_DIR`` environment variable, or
    None (unset, or not a directory).  Fixture generators, the checker build and the tests
    that read the reference's own files use it; there is no default location."""
    v = _os.environ.get("VDIT_REFERENCE_DIR")
    if not v:
        return None
    p = _Path(v)
    return p if p.is_dir() else None
