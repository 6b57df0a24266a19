"""Seeded synthetic inputs with the shapes of the benchmark configurations.

The reference is measured on the hackathon's cached voxel sets and DINOv3
features, which are not available here; these generators stand in with the
same shapes and value distributions:

* ``shell_voxels``     jittered sphere shell in a cubic grid (C1, C3, C4);
* ``uniform_voxels``   unique uniform cells (C2);
* ``ellipsoid_union``  union of 1-3 random ellipsoid shells (C5);
* ``C4``               the full 24-block DiT workload (N=16384, 64^3, r=36).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .model import LatDitArch


def shell_voxels(n: int, grid: int, radius: float, seed: int, jitter: float = 0.3) -> np.ndarray:
    """n unique voxels of a jittered one-voxel-thick sphere shell centred in the grid
    (points outside the grid are dropped), int32 [n,3]."""
    rng = np.random.default_rng(seed)
    pts = np.zeros((0, 3), dtype=np.int64)
    m = 8 * n
    c = (grid - 1) / 2.0
    for _ in range(8):
        d = rng.normal(size=(m, 3))
        d /= np.linalg.norm(d, axis=1, keepdims=True)
        p = np.rint(c + radius * d + rng.normal(scale=jitter, size=(m, 3))).astype(np.int64)
        p = p[np.all((p >= 0) & (p < grid), axis=1)]
        pts = np.unique(np.concatenate([pts, p]), axis=0)
        if len(pts) >= n:
            break
        jitter *= 1.5          # thicken the shell until it holds n voxels
    if len(pts) < n:
        raise ValueError(f"shell r={radius} in {grid}^3 holds only {len(pts)} voxels")
    return pts[rng.permutation(len(pts))[:n]].astype(np.int32)


def uniform_voxels(n: int, grid: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    c = rng.choice(grid ** 3, size=n, replace=False)
    return np.stack([c // (grid * grid), (c // grid) % grid, c % grid], -1).astype(np.int32)


def ellipsoid_union(n: int, grid: int, seed: int) -> np.ndarray:
    """Union of 1-3 random ellipsoid shells, topped up / subsampled to exactly n voxels."""
    rng = np.random.default_rng(seed)
    k = int(rng.integers(1, 4))
    pts = []
    for _ in range(k):
        ctr = rng.uniform(0.3 * grid, 0.7 * grid, size=3)
        ax = rng.uniform(0.15 * grid, 0.35 * grid, size=3)
        m = 6 * n
        d = rng.normal(size=(m, 3))
        d /= np.linalg.norm(d, axis=1, keepdims=True)
        pts.append(np.rint(ctr + ax * d + rng.normal(scale=0.3, size=(m, 3))).astype(np.int64))
    p = np.concatenate(pts)
    p = np.unique(p[np.all((p >= 0) & (p < grid), axis=1)], axis=0)
    if len(p) < n:
        extra = uniform_voxels(n, grid, seed + 1).astype(np.int64)
        p = np.unique(np.concatenate([p, extra]), axis=0)
    return p[rng.permutation(len(p))[:n]].astype(np.int32)


@dataclass
class C4:
    """Full DiT: 24 blocks, dim 1536, 12 x 128 heads, bf16 linears, fp32 ffn_conv,
    N=16384 voxels on a sphere shell (r=36) in 64^3, context [4101, 1536] N(0,1),
    4-step exact solver (3 guided at CFG 3.0 + 1 unguided = 7 NFE)."""
    n: int = 16384
    grid: int = 64
    radius: float = 36.0
    ctx_tokens: int = 4101
    guidance: float = 3.0

    arch = LatDitArch(dim=1536, head_dim=128, depth=24, cond_depth=8, res=64, patch_size=4096)

    def inputs(self, seed: int, device) -> dict:
        vox = torch.from_numpy(shell_voxels(self.n, self.grid, self.radius, seed))
        g = torch.Generator(device="cpu").manual_seed(seed + 1)
        ctx = torch.randn(self.ctx_tokens, self.arch.dim, generator=g)
        noise = torch.randn(self.n, self.arch.latent_dim, generator=g)
        dino = torch.randn(1, self.ctx_tokens, self.arch.dino_dim, generator=g).to(torch.float16)
        return {"vox": vox.to(device), "context": ctx.to(device, torch.bfloat16), "noise": noise.to(device),
                "vox_host": vox, "dino_host": dino, "noise_host": noise}


@dataclass
class C5:
    """Sharded batch: 16 independent samples, each N=32768 voxels from a seeded union of
    1-3 random ellipsoid shells in 128^3 with a [4101, 1536] N(0,1) context, through the
    same 24-block DiT (RoPE resolution 128) and 4-step exact solver as C4."""
    n: int = 32768
    grid: int = 128
    samples: int = 16
    ctx_tokens: int = 4101
    guidance: float = 3.0

    arch = LatDitArch(dim=1536, head_dim=128, depth=24, cond_depth=8, res=128, patch_size=4096)

    def inputs(self, seed: int, device) -> dict:
        vox = torch.from_numpy(ellipsoid_union(self.n, self.grid, seed))
        g = torch.Generator(device="cpu").manual_seed(seed + 1)
        ctx = torch.randn(self.ctx_tokens, self.arch.dim, generator=g)
        noise = torch.randn(self.n, self.arch.latent_dim, generator=g)
        return {"vox": vox.to(device), "context": ctx.to(device, torch.bfloat16), "noise": noise.to(device)}

