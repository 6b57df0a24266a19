"""The benchmark's on-disk inputs: a sample's voxel indices and its cached DINOv3 features,
read the way the reference's evaluation driver reads them
(``BK/scripts/hackathon/run_lat_dit_eval.py:95-135, 283-292``) and packed into the plugin's
call arguments (``Solution.generate(vox_idxs, conditioning=LatDitConditioning(...))``).

Layout of a sample directory (``<root>/<sample_id>[/cache]``): ``vox_idxi.npz`` (key
``vox_idxi``, or ``arr_0``: int32 ``[N, 3]``); ``<view>_dinov3.npz`` or ``dinov3.npz``
(keys ``feats`` fp16 ``[1, 4101, 1280]`` and ``token`` fp16 ``[1, 1280]``), or the older
``dinov3_feats.pt`` / ``dinov3_token.pt`` pair.  The default view is ``4view_000``.
Host-side only: the arrays stay in (optionally pinned) host memory; the plugin copies
them to the GPU and ``image_map`` maps the features there.
"""
from __future__ import annotations

from pathlib import Path
from typing import List, Tuple, Union

import numpy as np
import torch

from .runtime import LatDitConditioning

DEFAULT_VIEW = "4view_000"


def load_vox_idxi(path: Union[str, Path]) -> np.ndarray:
    """Voxel indices ``[N, 3]`` from ``vox_idxi.npz`` (key ``vox_idxi`` or ``arr_0``)."""
    with np.load(path) as data:
        for key in ("vox_idxi", "arr_0"):
            if key in data.files:
                vox = np.asarray(data[key])
                break
        else:
            raise KeyError(f"no voxel indices in {path}; keys={data.files}")
    if vox.ndim != 2 or vox.shape[1] != 3:
        raise ValueError(f"{path}: voxel indices must be [N, 3], got {vox.shape}")
    return vox


def load_dinov3(sample_cache_dir: Union[str, Path], view_name: str = DEFAULT_VIEW) -> Tuple[np.ndarray, np.ndarray]:
    """(feats, token) of one view: ``<view>_dinov3.npz``, else ``dinov3.npz``, else the
    ``dinov3_feats.pt`` / ``dinov3_token.pt`` pair."""
    d = Path(sample_cache_dir)
    for combined in (d / f"{view_name}_dinov3.npz", d / "dinov3.npz"):
        if combined.exists():
            with np.load(combined) as data:
                return np.asarray(data["feats"]), np.asarray(data["token"])
    feats_pt, token_pt = d / "dinov3_feats.pt", d / "dinov3_token.pt"
    if feats_pt.exists() and token_pt.exists():
        return (torch.load(feats_pt, map_location="cpu").numpy(), torch.load(token_pt, map_location="cpu").numpy())
    raise FileNotFoundError(f"missing DINOv3 cache in {d} (expected {view_name}_dinov3.npz, dinov3.npz or *.pt)")


def resolve_sample_cache_dir(sample_root: Union[str, Path]) -> Path:
    """``<sample_root>/cache`` when it exists, else the sample root itself."""
    root = Path(sample_root)
    return root / "cache" if (root / "cache").is_dir() else root


def load_sample(sample_root: Union[str, Path], view_name: str = DEFAULT_VIEW,
                pin_memory: bool = False) -> Tuple[List[torch.Tensor], LatDitConditioning]:
    """One sample as the plugin's call arguments: ``([vox int32 [N, 3]], conditioning)``
    with ``dino_features`` ``[1, 4101, 1280]`` and ``dino_token`` ``[1, 1280]`` (fp16, host)."""
    d = resolve_sample_cache_dir(sample_root)
    vox = torch.from_numpy(np.ascontiguousarray(load_vox_idxi(d / "vox_idxi.npz"), dtype=np.int32))
    feats, token = load_dinov3(d, view_name)
    feats_t = torch.from_numpy(np.ascontiguousarray(feats))
    token_t = torch.from_numpy(np.ascontiguousarray(token))
    if feats_t.dim() == 2:
        feats_t = feats_t.unsqueeze(0)
    if pin_memory:
        vox, feats_t, token_t = vox.pin_memory(), feats_t.pin_memory(), token_t.pin_memory()
    return [vox], LatDitConditioning(dino_features=feats_t, dino_token=token_t, batch_size=1)


def list_samples(cache_root: Union[str, Path], view_name: str = DEFAULT_VIEW) -> List[str]:
    """Sample ids under a cache root that hold the view's features (sorted, as the driver walks them)."""
    root = Path(cache_root)
    ids = []
    for p in sorted(root.iterdir()):
        if not p.is_dir():
            continue
        d = resolve_sample_cache_dir(p)
        if (d / f"{view_name}_dinov3.npz").is_file() or (d / "dinov3.npz").is_file() or \
                (d / "dinov3_feats.pt").is_file():
            ids.append(p.name)
    return ids
