"""Inputs of the full-size parity cases, shared by the fixture generator
(``make_golden_full.py``, which runs the reference on CPU) and the GPU tests.

Every tensor is rebuilt from a seed on the CPU, so the fixtures hold only the
reference's outputs and a few checksums of the rebuilt inputs (a test first
checks the checksums, so a host that rebuilds different inputs fails loudly
instead of reporting a parity error).

Cases, with the benchmark's shapes and value distributions:

* ``c1``        one context block (depth 1, cond_depth 1), dim 1536, 12 x 128 heads,
                N = 4096 voxels of a jittered sphere shell (r = 24) in 64^3,
                context [4101, 1536] N(0,1), xt [N, 16] N(0,1), t = 0.5;
                weights N(0, 0.02), biases 0, norm gains 1.  Both branches.
* ``c4nfe_128`` / ``c4nfe_96``
                one NFE of a depth-2 model (one context block, one plain block) at
                the full width and context: dim 1536, 12 x 128 or 16 x 96 heads,
                N = 16384 on the r = 36 shell in 64^3, 4101 context tokens, t = 0.75.
* ``c4sample``  the full model (24 blocks, 8 with context, 12 x 128) through the exact
                4-step sampler (t = 1, .9, .75, .5, 0; three guided steps at CFG 3.0
                with the 1-token unconditional branch, one unguided): 7 NFEs on
                N = 16384, DINO features [1, 4101, 1280] N(0,1) mapped by image_map.
"""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


@dataclass(frozen=True)
class Case:
    name: str
    dim: int
    head_dim: int
    depth: int
    cond_depth: int
    n: int
    radius: float
    weight_seed: int
    input_seed: int
    t: float = 0.5
    ctx_tokens: int = 4101
    grid: int = 64

    def arch(self):
        from vdit.model import LatDitArch
        return LatDitArch(dim=self.dim, head_dim=self.head_dim, depth=self.depth, cond_depth=self.cond_depth,
                          res=self.grid, patch_size=4096)

    def model_config(self) -> dict:
        return self.arch().model_config()

    def weights(self) -> dict:
        """Seeded CPU weights: linears and conv N(0, 0.02), biases 0, gains 1."""
        from vdit.model import LatDitModel
        return LatDitModel.random(self.arch(), seed=self.weight_seed).state

    def voxels(self) -> np.ndarray:
        from vdit.workloads import shell_voxels
        return shell_voxels(self.n, self.grid, self.radius, self.input_seed)

    def nfe_inputs(self):
        """(xt [N, 16] in input voxel order, context [L, D]) for the one-NFE cases."""
        g = torch.Generator().manual_seed(self.input_seed + 1)
        xt = torch.randn(self.n, 16, generator=g)
        ctx = torch.randn(self.ctx_tokens, self.dim, generator=g)
        return xt, ctx

    def sample_inputs(self):
        """(DINO features [1, L, 1280], noise [N, 16]) for the sampler case; the noise is
        the draw the reference's sampler makes from ``torch.Generator().manual_seed(noise_seed)``."""
        g = torch.Generator().manual_seed(self.input_seed + 1)
        dino = torch.randn(1, self.ctx_tokens, 1280, generator=g)
        noise = torch.randn(self.n, 16, generator=torch.Generator().manual_seed(self.noise_seed))
        return dino, noise

    @property
    def noise_seed(self) -> int:
        return self.input_seed + 2

    def fixture_path(self) -> Path:
        return HERE / f"{self.name}.npz"


CASES = {
    "c1": Case("c1", 1536, 128, 1, 1, 4096, 24.0, weight_seed=1001, input_seed=1002, t=0.5),
    "c4nfe_128": Case("c4nfe_128", 1536, 128, 2, 1, 16384, 36.0, weight_seed=1011, input_seed=1012, t=0.75),
    "c4nfe_96": Case("c4nfe_96", 1536, 96, 2, 1, 16384, 36.0, weight_seed=1021, input_seed=1022, t=0.75),
    "c4sample": Case("c4sample", 1536, 128, 24, 8, 16384, 36.0, weight_seed=1031, input_seed=1032),
}


def checksums(tensors: dict) -> np.ndarray:
    """float64 sums of |x| of the named tensors, in sorted key order."""
    return np.array([float(tensors[k].double().abs().sum()) for k in sorted(tensors)], dtype=np.float64)


def weight_checksum(state: dict) -> float:
    """One float64 number over every weight tensor (sum of |x|, keys in sorted order)."""
    return float(sum(float(state[k].double().abs().sum()) for k in sorted(state)))


def load(name: str) -> dict:
    return dict(np.load(CASES[name].fixture_path()))
