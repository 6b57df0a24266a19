"""``Solution(LatDitGenerator)``: the plugin the lat_dit harness loads.

Same contract as the reference's ``solution.py:135-246``:
``from_pretrained(path, device=None, torch_dtype=None, **kw)`` discovers the
weights (``path``, ``path/lat_dit``, ``$LAT_DIT_DIR``, ``$LAT_DIT_WEIGHTS_DIR``,
``$KANDI3D_WEIGHTS_DIR``, ``--lat-dit-dir`` on argv, ``solution.py:48-102``),
loads config + solver config, builds the runner and warms it up;
``generate_impl`` returns one [N_i, 16] fp32 latent tensor per sample, in the
caller's voxel order.  ``generate()`` is inherited and never overridden.
Batches run sample by sample (each sample owns its geometry).
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path
from typing import Any, Optional, Union

import torch

from .fast_flow import OptimizedLatDitRunner
from .fast_sampler import SolverConfig
from .model import LatDitModel
from .runtime import FlowMatchSamplingParams, LatDitConditioning, LatDitGenerator, resolve


def _has_weights(d: Path) -> bool:
    return (d / "diffusion_pytorch_model.safetensors").is_file() or (d / "diffusion_pytorch_model.bin").is_file()


def _discover_weights_dir(primary: Path) -> Path:
    cands = [primary, primary / "lat_dit"]
    argv = sys.argv
    if "--lat-dit-dir" in argv:
        i = argv.index("--lat-dit-dir")
        if i + 1 < len(argv):
            cands.append(Path(argv[i + 1]))
    for env in ("LAT_DIT_DIR", "LAT_DIT_WEIGHTS_DIR", "KANDI3D_WEIGHTS_DIR"):
        if os.environ.get(env):
            p = Path(os.environ[env])
            cands += [p, p / "lat_dit"]
    for c in cands:
        if _has_weights(c):
            return c
    return primary


class Solution(LatDitGenerator):
    """B200 lat_dit generator: exact Euler+CFG sampler with the 1-token uncond branch."""

    def __init__(self, inner: LatDitModel, solver_config: Optional[SolverConfig] = None,
                 weights_dir: Optional[Path] = None, device: Optional[torch.device] = None,
                 cuda_graph: bool = False):
        self.inner = inner
        self.solver_config = solver_config or SolverConfig()
        sc = self.solver_config
        self._default_runtime = FlowMatchSamplingParams(guidance_scale=sc.guidance_scale, cfg_range=sc.cfg_range,
                                                        rescale_t=sc.rescale_t,
                                                        num_inference_steps=sc.num_inference_steps)
        self.runner = OptimizedLatDitRunner(inner, sc, weights_dir=weights_dir, device=device, cuda_graph=cuda_graph)

    @classmethod
    def from_pretrained(cls, pretrained_model_name_or_path: Union[str, os.PathLike],
                        device: Optional[Union[torch.device, str, int]] = None,
                        torch_dtype: Optional[torch.dtype] = None, **kwargs: Any) -> "Solution":
        primary = Path(pretrained_model_name_or_path).expanduser().resolve()
        wdir = _discover_weights_dir(primary)
        cfg_dir = primary if (primary / "config.json").is_file() else wdir
        cfg = json.loads((cfg_dir / "config.json").read_text(encoding="utf-8"))
        mc = dict(cfg.get("model_config", cfg))
        if "latent_scale" in cfg:
            mc.setdefault("latent_scale", cfg["latent_scale"])
        model = LatDitModel.from_pretrained(wdir) if _has_weights(wdir) else None
        if model is None:
            raise FileNotFoundError(f"no diffusion_pytorch_model.safetensors or .bin found for {primary}")
        solver = SolverConfig.from_dir(primary, fallback_model_cfg=mc)
        if device is not None:
            device = torch.device(f"cuda:{device}" if isinstance(device, int) else device)
        inst = cls(model, solver_config=solver, weights_dir=primary, device=device,
                   cuda_graph=bool(kwargs.get("cuda_graph", False)))
        if solver.warmup_on_load:
            inst.runner.warmup()
        return inst

    def parameters(self, recurse: bool = True):
        return self.inner.parameters(recurse)

    def to(self, *args: Any, **kwargs: Any) -> "Solution":
        dev = kwargs.get("device", args[0] if args else None)
        if dev is not None:
            self.runner = OptimizedLatDitRunner(self.inner, self.solver_config, self.runner.weights_dir,
                                                device=torch.device(dev), cuda_graph=self.runner.cuda_graph)
        return self

    def eval(self) -> "Solution":
        return self

    @torch.no_grad()
    def generate_impl(self, vox_idxs: list, *, conditioning: LatDitConditioning,
                      sampling: Optional[FlowMatchSamplingParams] = None, generator: Optional[torch.Generator] = None,
                      **sampling_kwargs: Any) -> list:
        resolved = resolve(self._default_runtime, sampling, **sampling_kwargs)
        dev = self.runner.device
        dino = conditioning.dino_features
        outs = []
        for i, vox in enumerate(vox_idxs):
            d_i = dino[i:i + 1] if dino.shape[0] > 1 else dino
            cond_i = LatDitConditioning(dino_features=d_i.to(dev, non_blocking=True), batch_size=1)
            outs += self.runner.sample_fast([vox.to(dev, non_blocking=True)], cond_i, sampling=resolved,
                                            generator=generator)
        return outs


__all__ = ["Solution"]
