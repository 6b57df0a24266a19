"""Multi-GPU plumbing of the sampler: one process per GPU, samples sharded
across ranks, latents gathered to rank 0; for fewer samples than GPUs, the two
branches of a guided step split over two ranks (``branch_split_steps``).

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


def branch_split_steps(xt: torch.Tensor, tl: Sequence[float], guided: Sequence[bool], g_scale: float, nfe, cfg_euler,
                       group=None) -> torch.Tensor:
    """The sampler's Euler + CFG loop for ONE sample on TWO ranks, for runs with fewer
    samples than GPUs (the reference runs both branches of a guided step on one GPU,
    ``lib/fast_flow.py:2836,2887,3288``).

    In a guided step, group rank 0 runs the conditional NFE and rank 1 the unconditional
    one at the same time.  The two ``[N, C]`` velocities are all-gathered, and both ranks
    apply the same CFG + Euler update, so ``xt`` stays identical on both.  In an unguided
    step rank 0 runs the NFE and broadcasts its velocity.
    ``nfe(x, t, uncond) -> v`` and ``cfg_euler(x, v, v_uncond or None, g, dt)`` (in place)
    are the caller's.  Every rank takes the same collective steps in the same order."""
    if dist.get_world_size(group) != 2:
        raise ValueError("the branch split runs on exactly two ranks")
    rank = dist.get_rank(group)
    src = dist.get_global_rank(group, 0) if group is not None else 0
    for i in range(len(guided)):
        dt = float(tl[i]) - float(tl[i + 1])
        if guided[i] and g_scale > 0:
            v_mine = nfe(xt, tl[i], rank == 1).contiguous()
            vs = [torch.empty_like(v_mine) for _ in range(2)]
            dist.all_gather(vs, v_mine, group=group)
            cfg_euler(xt, vs[0], vs[1], g_scale, dt)
        else:
            v = nfe(xt, tl[i], False).contiguous() if rank == 0 else torch.empty_like(xt)
            dist.broadcast(v, src=src, group=group)
            cfg_euler(xt, v, None, g_scale, dt)
    return xt
