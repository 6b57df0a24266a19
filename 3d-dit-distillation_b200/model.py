"""Weights and architecture of the lat_dit ``FlowModel`` as the runner consumes them.

``LatDitModel`` holds the checkpoint tensors under the reference key names
(``flow.blocks.{i}.to_qkv.weight``, ``image_map.weight``, ``mean``, ``std``;
see ``BK/kandi3d_image23d/models/modeling_lat_dit.py`` and the lat_dit
safetensors header) plus the architecture fields of ``weights/config.json``
``model_config``.  It loads ``diffusion_pytorch_model.safetensors``/``.bin``,
strips ``_orig_mod.`` prefixes like ``normalize_state_dict``
(``BK/kandi3d_image23d/modeling_utils.py:11-12``), or builds seeded random
weights for synthetic runs.
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Dict, Optional, Sequence

import torch

ORDERS = ("h", "ht1", "h1", "ht")


@dataclass
class LatDitArch:
    dim: int = 1536
    head_dim: int = 96
    depth: int = 24
    cond_depth: int = 8
    ffn_rate: float = 2.5
    res: int = 64
    latent_dim: int = 16
    latent_scale: float = 1.5
    patch_size: int = 4096
    time_pos_features: int = 256
    dino_dim: int = 1280
    orders: Sequence[str] = ORDERS
    cfg: float = 7.0
    cfg_range: tuple = (0.5, 1.0)
    rescale_t: float = 3.0
    num_inference_steps: int = 14

    @property
    def heads(self) -> int:
        return self.dim // self.head_dim

    @property
    def ffn_dim(self) -> int:
        return int(self.dim * self.ffn_rate)

    @classmethod
    def from_model_config(cls, mc: Dict) -> "LatDitArch":
        a = cls()
        for k in ("dim", "head_dim", "depth", "cond_depth", "ffn_rate", "res", "latent_dim", "latent_scale",
                  "patch_size", "time_pos_features", "cfg", "rescale_t", "num_inference_steps"):
            if k in mc:
                setattr(a, k, type(getattr(a, k))(mc[k]))
        if "orders" in mc:
            a.orders = tuple(mc["orders"])
        if "cfg_range" in mc:
            a.cfg_range = tuple(float(x) for x in mc["cfg_range"])
        for flag, want in (("io_conv", False), ("pos_conv", False), ("patch", 1), ("rope", True), ("rms", True),
                           ("ffn_conv", True), ("clf_shared", False), ("use_token", False), ("pos_emb", False)):
            if flag in mc and mc[flag] != want:
                raise NotImplementedError(f"model_config {flag}={mc[flag]!r}: this path is built for {want!r}")
        return a

    def model_config(self) -> Dict:
        return {"dim": self.dim, "head_dim": self.head_dim, "depth": self.depth, "cond_depth": self.cond_depth,
                "ffn_rate": self.ffn_rate, "res": self.res, "latent_dim": self.latent_dim,
                "latent_scale": self.latent_scale, "patch_size": self.patch_size, "orders": list(self.orders),
                "cfg": self.cfg, "cfg_range": list(self.cfg_range), "rescale_t": self.rescale_t,
                "num_inference_steps": self.num_inference_steps}


def param_shapes(a: LatDitArch) -> Dict[str, tuple]:
    """Checkpoint key -> shape (lat_dit safetensors header)."""
    D, F2, Fh, L, H, HD = a.dim, 2 * a.ffn_dim, a.ffn_dim, a.latent_dim, a.heads, a.head_dim
    s = {"image_map.weight": (D, a.dino_dim), "image_map.bias": (D,),
         "flow.time_embed.0.weight": (4 * D, a.time_pos_features), "flow.time_embed.0.bias": (4 * D,),
         "flow.time_embed.2.weight": (D, 4 * D), "flow.time_embed.2.bias": (D,),
         "flow.patchify.weight": (D, L), "flow.unpatchify.weight": (L, D),
         "flow.out_gates.weight": (2 * D, D), "flow.out_gates.bias": (2 * D,), "mean": (L,), "std": (L,)}
    for b in range(a.depth):
        p = f"flow.blocks.{b}."
        lin = {"gates": (9 * D, D), "to_qkv": (3 * D, D), "to_out": (D, D), "to_out_cross": (D, D),
               "ffn0": (F2, D), "ffn1": (D, Fh)}
        if b < a.cond_depth:
            lin.update({"cond_gates": (9 * D, D), "cond_to_qkv": (3 * D, D), "cond_to_out": (D, D),
                        "to_qkv_cross": (3 * D, D), "cond_to_qkv_cross": (3 * D, D), "cond_to_out_cross": (D, D),
                        "cond_ffn0": (F2, D), "cond_ffn1": (D, Fh)})
        else:
            lin.update({"to_q_cross": (D, D), "cond_gates": (2 * D, D), "cond_to_kv_cross": (2 * D, D)})
        for n, sh in lin.items():
            s[p + n + ".weight"] = sh
            s[p + n + ".bias"] = (sh[0],)
        s[p + "ffn_conv.weight"] = (3, 3, 3, F2)
        s[p + "ffn_conv.bias"] = (F2,)
        s[p + "qk_norm.q_scale"] = (H, HD)
        s[p + "qk_norm.k_scale"] = (H, HD)
        if b < a.cond_depth:
            s[p + "cond_qk_norm.q_scale"] = (H, HD)
            s[p + "cond_qk_norm.k_scale"] = (H, HD)
    return s


class LatDitModel:
    """Checkpoint tensors + architecture.  ``state`` values stay where they were
    loaded (CPU fp32 for checkpoints); the runner makes its own device copies."""

    def __init__(self, arch: LatDitArch, state: Dict[str, torch.Tensor]):
        self.arch = arch
        self.state = state
        missing = [k for k in param_shapes(arch) if k not in state]
        if missing:
            raise KeyError(f"state dict misses {len(missing)} keys, e.g. {missing[:3]}")

    # reference-compatible accessors
    @property
    def latent_scale(self) -> float:
        return self.arch.latent_scale

    def state_dict(self) -> Dict[str, torch.Tensor]:
        return self.state

    def parameters(self, recurse: bool = True):
        return iter(self.state.values())

    @classmethod
    def from_state_dict(cls, state: Dict[str, torch.Tensor], model_config: Dict) -> "LatDitModel":
        sd = {}
        for k, v in state.items():
            k = k.replace("_orig_mod.", "")
            if k.startswith("core."):
                k = k[5:]
            sd[k] = v
        return cls(LatDitArch.from_model_config(model_config), sd)

    @classmethod
    def from_pretrained(cls, path) -> "LatDitModel":
        path = Path(path)
        cfg = json.loads((path / "config.json").read_text(encoding="utf-8"))
        mc = cfg.get("model_config", cfg)
        st = path / "diffusion_pytorch_model.safetensors"
        if st.is_file():
            from safetensors.torch import load_file
            sd = load_file(str(st))
        else:
            b = path / "diffusion_pytorch_model.bin"
            if not b.is_file():
                raise FileNotFoundError(f"no diffusion_pytorch_model.safetensors or .bin in {path}")
            sd = torch.load(b, map_location="cpu", weights_only=True)
        if "latent_scale" in cfg and "latent_scale" not in mc:
            mc = dict(mc, latent_scale=cfg["latent_scale"])
        return cls.from_state_dict(sd, mc)

    @classmethod
    def random(cls, arch: LatDitArch, seed: int = 0, weight_std: float = 0.02,
               device: Optional[torch.device] = None) -> "LatDitModel":
        """Seeded synthetic weights: linears and conv N(0, weight_std), biases 0,
        q/k gains 1, mean 0, std 1 (the synthetic-benchmark initialisation)."""
        g = torch.Generator(device=device if device is not None else "cpu").manual_seed(seed)
        sd = {}
        for k, sh in sorted(param_shapes(arch).items()):
            if k == "std" or k.endswith("_scale"):
                t = torch.ones(sh, device=device)
            elif k == "mean" or k.endswith(".bias"):
                t = torch.zeros(sh, device=device)
            else:
                t = torch.randn(sh, generator=g, device=device) * weight_std
            sd[k] = t
        return cls(arch, sd)
