"""Multi-GPU plumbing of the sampler: one process per GPU, samples sharded
across ranks, latents gathered to rank 0.

Samples are independent (each owns its geometry and its 7 NFEs), so the forward
has no collective; the only exchange is the end-of-run gather of the
variable-length ``[N_i, 16]`` fp32 latents: sizes first (all-gather), then a
padded gather to the destination rank — the pattern of the reference's
``BK/base_models/optimization_utils.py:511-535`` (``all_gather_image``).
Works with NCCL (GPU tensors) and gloo (CPU tensors, used by the tests).
"""
from __future__ import annotations

import datetime
import os
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist


def init_from_env(backend: str = "nccl", timeout_s: float = 120.0):
    """Initialise the default process group from torchrun's environment.
    Returns (rank, world_size, local_rank); a single process returns (0, 1, 0)
    without a process group."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return 0, 1, 0
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    kw = {}
    if backend == "nccl":
        torch.cuda.set_device(local)
        kw["device_id"] = torch.device("cuda", local)
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank, world, local


def shard_samples(n_samples: int, rank: int, world: int) -> List[int]:
    """Round-robin sample indices owned by ``rank``."""
    return list(range(rank, n_samples, world))


def gather_latents(latents: Sequence[torch.Tensor], rank: int, world: int,
                   dst: int = 0) -> Optional[List[torch.Tensor]]:
    """Gather every rank's list of ``[N_i, C]`` tensors to ``dst``.

    Each rank contributes the same number of tensors (pad with empty tensors if
    the shards are uneven).  Returns the list of ``world * len(latents)`` tensors,
    rank-major, on ``dst``; None elsewhere."""
    if world == 1:
        return list(latents)
    dev = latents[0].device if latents else torch.device("cpu")
    k = len(latents)
    c = latents[0].shape[1] if latents else 16
    sizes = torch.tensor([t.shape[0] for t in latents], dtype=torch.int64, device=dev)
    all_sizes = [torch.empty_like(sizes) for _ in range(world)]
    dist.all_gather(all_sizes, sizes)
    mx = max(int(s.max()) if s.numel() else 0 for s in all_sizes)
    pad = torch.zeros(k, max(mx, 1), c, dtype=latents[0].dtype if latents else torch.float32, device=dev)
    for i, t in enumerate(latents):
        pad[i, : t.shape[0]] = t
    outs = [torch.empty_like(pad) for _ in range(world)] if rank == dst else None
    dist.gather(pad, outs, dst=dst)
    if rank != dst:
        return None
    res = []
    for r in range(world):
        for i in range(k):
            res.append(outs[r][i, : int(all_sizes[r][i])])
    return res
