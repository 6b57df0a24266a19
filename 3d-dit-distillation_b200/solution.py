"""``Solution(LatDitGenerator)``: the plugin the lat_dit harness loads.

Same contract as the reference's ``solution.py:135-246``:
``from_pretrained(path, device=None, torch_dtype=None, **kw)`` discovers the
weights in the reference's order (``solution.py:48-102``), loads config + solver
config, folds a distilled adapter found beside the weights into them
(``solution.py:105-132``, called at ``:205``), builds the runner and warms it up;
``generate_impl`` returns one [N_i, 16] fp32 latent tensor per sample, in the
caller's voxel order.  ``generate()`` is inherited and never overridden.
Batches run sample by sample (each sample owns its geometry).
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path
from typing import Any, Dict, Optional, Sequence, Union

import torch

from .fast_flow import OptimizedLatDitRunner
from .fast_sampler import SolverConfig
from .model import LatDitModel
from .runtime import FlowMatchSamplingParams, LatDitConditioning, LatDitGenerator, resolve

# Organiser locations the reference tries last, relative to the working directory
# unless absolute (``solution.py:91-100``).
DEFAULT_WEIGHT_LOCATIONS = ("weights/lat_dit", "kandi3d_weights_aijc_kit/lat_dit", "../weights/lat_dit",
                            "/weights/lat_dit", "/workspace/weights/lat_dit")


def _has_weights(d: Path) -> bool:
    return (d / "diffusion_pytorch_model.safetensors").is_file() or (d / "diffusion_pytorch_model.bin").is_file()


def _dir_or_lat_dit(c: Path) -> Optional[Path]:
    if _has_weights(c):
        return c
    if _has_weights(c / "lat_dit"):
        return c / "lat_dit"
    return None


def _discover_weights_dir(primary: Path, argv: Optional[Sequence[str]] = None,
                          environ: Optional[Dict[str, str]] = None) -> Path:
    """The directory holding ``diffusion_pytorch_model.safetensors`` (or ``.bin``), searched
    in the reference's order (``solution.py:48-102``): ``primary`` and ``primary/lat_dit``;
    then, scanning the command line, ``--lat-dit-dir X`` / ``--lat-dit-dir=X`` (X or
    X/lat_dit) and ``--lat-vae-dir X`` / ``--lat-vae-dir=X`` (the ``lat_dit`` directory beside
    X); then ``$LAT_DIT_DIR``, ``$LAT_DIT_WEIGHTS_DIR``, ``$KANDI3D_WEIGHTS_DIR`` (each as is
    or its ``lat_dit``); then the organiser locations.  Falls back to ``primary``."""
    argv = sys.argv if argv is None else argv
    environ = os.environ if environ is None else environ
    hit = _dir_or_lat_dit(primary)
    if hit is not None:
        return hit
    for i, arg in enumerate(argv):
        if arg == "--lat-dit-dir" and i + 1 < len(argv):
            hit = _dir_or_lat_dit(Path(argv[i + 1]).expanduser().resolve())
        elif arg.startswith("--lat-dit-dir="):
            hit = _dir_or_lat_dit(Path(arg.split("=", 1)[1]).expanduser().resolve())
        elif arg == "--lat-vae-dir" and i + 1 < len(argv):
            c = Path(argv[i + 1]).expanduser().resolve().parent / "lat_dit"
            hit = c if _has_weights(c) else None
        elif arg.startswith("--lat-vae-dir="):
            c = Path(arg.split("=", 1)[1]).expanduser().resolve().parent / "lat_dit"
            hit = c if _has_weights(c) else None
        if hit is not None:
            return hit
    for env in ("LAT_DIT_DIR", "LAT_DIT_WEIGHTS_DIR", "KANDI3D_WEIGHTS_DIR"):
        v = environ.get(env)
        if v:
            hit = _dir_or_lat_dit(Path(v).expanduser().resolve())
            if hit is not None:
                return hit
    for rel in DEFAULT_WEIGHT_LOCATIONS:
        if _has_weights(Path(rel)):
            return Path(rel).resolve()
    return primary


def merge_distilled_adapters(state: Dict[str, torch.Tensor], custom_dir: Path) -> int:
    """Fold a distilled adapter (``custom_dir/student_adapter.pt``) into the checkpoint
    tensors, as the reference does at load (``solution.py:105-132``): for every LoRA pair
    ``W += (B @ A) * lora_scale`` (``lora_scale`` default 1), then ``W += delta`` for every
    entry of ``weight_deltas``; keys absent from the checkpoint are skipped, an unreadable
    file is ignored.  The sums are taken in fp32 and the folded tensors stay fp32 (the
    reference's parameters are fp32).  Returns the number of tensors changed."""
    adapter = Path(custom_dir) / "student_adapter.pt"
    if not adapter.is_file():
        return 0
    try:
        payload = torch.load(adapter, map_location="cpu", weights_only=True)
    except Exception:          # the reference ignores an adapter it cannot read
        return 0
    changed = 0
    scale = float(payload.get("lora_scale", 1.0))
    lora_b = payload.get("lora_B", {})
    for key, a in payload.get("lora_A", {}).items():
        b = lora_b.get(key)
        if b is not None and key in state:
            w = state[key]
            state[key] = w.float() + ((b.float() @ a.float()) * scale).to(w.device)
            changed += 1
    for key, delta in payload.get("weight_deltas", {}).items():
        if key in state:
            w = state[key]
            state[key] = w.float() + delta.float().to(w.device)
            changed += 1
    return changed


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
        merge_distilled_adapters(model.state, primary)
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


__all__ = ["Solution", "merge_distilled_adapters"]
