"""Sampler surface of the reference's ``lib/fast_sampler.py`` (exact subset).

``SolverConfig`` keeps the reference's field names; only the exact solver is
built (piecewise Euler aligned to the CFG threshold, exact CFG every guided
step, exact 1-token unconditional branch).  The reference's calibrated
approximations (QAOA readout, cross-step caches) are not part of this path:
their fields are read and ignored, and ``approximate_fields_ignored`` lists
any that a loaded config switched on.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field, fields
from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple

import torch


@dataclass
class SolverConfig:
    num_inference_steps: int = 4
    n_guided_steps: int = 3
    n_unguided_steps: int = 1
    guidance_scale: float = 7.0
    cfg_range: Tuple[float, float] = (0.5, 1.0)
    rescale_t: float = 3.0
    solver_type: str = "piecewise_euler"      # "euler" | "piecewise_euler"
    cfg_stride: int = 1
    cfg_cache_mode: str = "exact"
    uncond_1token_condensation: bool = True
    ditfastattn_b0_msa_share: bool = True      # exact: block-0 self-attn is branch-independent
    qaoa_enabled: bool = False
    mid_block_cache_enabled: bool = False
    use_bf16_weights: bool = True
    use_fused_triton_kernels: bool = True     # name kept; the kernels here are CUDA
    precompute_rope_tables: bool = True
    precompute_time_gates: bool = True
    warmup_on_load: bool = True
    eval_cond_steps: List[int] = field(default_factory=list)
    eval_uncond_steps: List[int] = field(default_factory=list)
    # the approximate CFG cache ("neg_reuse"), opt-in; the reference's defaults
    # (lib/fast_sampler.py:25-79) apply once cfg_cache_mode is "neg_reuse"
    cfg_zero_star_projection: bool = True
    autotarget_clean_endpoint_blend: float = 0.08
    fastercache_freq_decoupled_cfg: bool = True
    fastercache_hf_boost: float = 0.035
    approximate_fields_ignored: List[str] = field(default_factory=list)

    _APPROX_FLAGS = ("qaoa_enabled", "mid_block_cache_enabled")

    @property
    def approximate_cfg_cache(self) -> bool:
        """True when guided steps may reuse the last unconditional velocity."""
        return self.cfg_cache_mode == "neg_reuse"

    def enable_approximate_cfg_cache(self, eval_uncond_steps: Optional[List[int]] = None,
                                     cfg_stride: int = 2) -> "SolverConfig":
        """Switch on the reference's default approximate CFG cache (``cfg_cache_mode
        "neg_reuse"``, unconditional NFE only at ``eval_uncond_steps``, default [0, 2])."""
        self.cfg_cache_mode = "neg_reuse"
        self.cfg_stride = int(cfg_stride)
        self.eval_uncond_steps = list(eval_uncond_steps) if eval_uncond_steps is not None else [0, 2]
        return self

    @classmethod
    def from_dir(cls, weights_dir: Optional[Path] = None,
                 fallback_model_cfg: Optional[Dict[str, Any]] = None,
                 allow_approximate_cfg_cache: bool = False) -> "SolverConfig":
        """Defaults <- model config (cfg, cfg_range, rescale_t) <- weights_dir/solver_config.json
        <- env LAT_DIT_STEPS / LAT_DIT_SOLVER (``lib/fast_sampler.py:163-203``).  A config that
        asks for the approximate CFG cache ("neg_reuse", cfg_stride, eval_uncond_steps) keeps it
        only with ``allow_approximate_cfg_cache``; otherwise it is listed as ignored."""
        cfg = cls()
        if fallback_model_cfg:
            if "cfg" in fallback_model_cfg:
                cfg.guidance_scale = float(fallback_model_cfg["cfg"])
            if "cfg_range" in fallback_model_cfg:
                cr = fallback_model_cfg["cfg_range"]
                cfg.cfg_range = (float(cr[0]), float(cr[1]))
            if "rescale_t" in fallback_model_cfg:
                cfg.rescale_t = float(fallback_model_cfg["rescale_t"])
        names = {f.name for f in fields(cls)}
        if weights_dir is not None:
            p = Path(weights_dir) / "solver_config.json"
            if p.is_file():
                data = json.loads(p.read_text(encoding="utf-8"))
                for k, v in data.items():
                    if k not in names or k == "approximate_fields_ignored":
                        continue
                    if k in cls._APPROX_FLAGS and v:
                        cfg.approximate_fields_ignored.append(k)
                        continue
                    if k == "solver_type" and v not in ("euler", "piecewise_euler"):
                        cfg.approximate_fields_ignored.append(f"solver_type={v}")
                        continue
                    approx_ok = allow_approximate_cfg_cache and data.get("cfg_cache_mode") == "neg_reuse"
                    if k == "cfg_cache_mode" and v != "exact" and not (approx_ok and v == "neg_reuse"):
                        cfg.approximate_fields_ignored.append(f"cfg_cache_mode={v}")
                        continue
                    if k == "cfg_stride" and int(v) != 1 and not approx_ok:
                        cfg.approximate_fields_ignored.append(f"cfg_stride={v}")
                        continue
                    if k == "eval_uncond_steps" and v and not approx_ok:
                        cfg.approximate_fields_ignored.append(f"eval_uncond_steps={v}")
                        continue
                    setattr(cfg, k, (float(v[0]), float(v[1])) if k == "cfg_range" else v)
        if "LAT_DIT_STEPS" in os.environ:
            steps = int(os.environ["LAT_DIT_STEPS"])
            cfg.num_inference_steps = steps
            cfg.n_guided_steps = max(1, int(round(steps * 0.75)))
            cfg.n_unguided_steps = max(1, steps - cfg.n_guided_steps)
        if os.environ.get("LAT_DIT_SOLVER") in ("euler", "piecewise_euler"):
            cfg.solver_type = os.environ["LAT_DIT_SOLVER"]
        return cfg


def build_schedule(solver_cfg: SolverConfig, num_steps_override: Optional[int] = None,
                   rescale_t_override: Optional[float] = None,
                   cfg_range_override: Optional[Tuple[float, float]] = None,
                   device: Optional[torch.device] = None) -> Tuple[torch.Tensor, List[bool], int]:
    """(t_seq [K+1], is_guided [K], n_guided), ``lib/fast_sampler.py:670-732`` without the QAOA branch."""
    r = rescale_t_override if rescale_t_override is not None else solver_cfg.rescale_t
    cr = cfg_range_override if cfg_range_override is not None else solver_cfg.cfg_range
    k = num_steps_override if num_steps_override is not None else solver_cfg.num_inference_steps

    def warp(u):
        return r * u / (1.0 + (r - 1.0) * u)

    if solver_cfg.solver_type == "euler":
        t = warp(torch.linspace(1.0, 0.0, k + 1, dtype=torch.float32, device=device))
        tl = t.tolist()
        g = [cr[0] <= tl[i] <= cr[1] for i in range(k)]
        return t, g, sum(g)
    t_low = float(cr[0])
    if 0.0 < t_low < 1.0 and k >= 2:
        u_low = t_low / (r - (r - 1.0) * t_low)
        if num_steps_override is not None and num_steps_override != solver_cfg.num_inference_steps:
            ng = max(1, int(round(k * (1.0 - u_low))))
            nu = max(1, k - ng)
        else:
            ng, nu = solver_cfg.n_guided_steps, solver_cfg.n_unguided_steps
            if ng + nu != k:
                ng = max(1, int(round(k * (1.0 - u_low))))
                nu = max(1, k - ng)
        ug = torch.linspace(1.0, u_low, ng + 1, dtype=torch.float32, device=device)
        uu = torch.linspace(u_low, 0.0, nu + 1, dtype=torch.float32, device=device)
        t = warp(torch.cat([ug[:-1], uu]))
        return t, [True] * ng + [False] * nu, ng
    t = warp(torch.linspace(1.0, 0.0, k + 1, dtype=torch.float32, device=device))
    tl = t.tolist()
    g = [cr[0] <= tl[i] <= cr[1] for i in range(k)]
    return t, g, sum(g)


def get_qaoa_eval_timesteps(solver_cfg: SolverConfig, t_list: List[float]) -> List[float]:
    """Evaluation times of each step: the step's own t (no QAOA shifts in the exact solver)."""
    return [float(t_list[i]) for i in range(len(t_list) - 1)]


def should_eval_uncond(step_idx: int, n_guided: int, cfg_stride: int, cfg_cache_mode: str,
                       eval_uncond_steps: Optional[List[int]] = None) -> bool:
    """``lib/fast_sampler.py:754-768``; always True for the exact solver."""
    if eval_uncond_steps:
        return step_idx in eval_uncond_steps
    if cfg_stride <= 1 or cfg_cache_mode == "exact":
        return True
    if step_idx == 0 or step_idx == n_guided - 1:
        return True
    return step_idx % cfg_stride == 0


def should_eval_cond(step_idx: int, n_guided: int, cond7_stride: int,
                     eval_cond_steps: Optional[List[int]] = None) -> bool:
    """``lib/fast_sampler.py:771-784``."""
    if step_idx == 0:
        return True
    if eval_cond_steps:
        return step_idx in eval_cond_steps
    if cond7_stride <= 1:
        return True
    return step_idx % cond7_stride == 0
