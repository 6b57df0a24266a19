"""Generate golden fixtures by running the reference implementation on CPU.

Usage (needs the reference checkout, read-only, and no GPU):

    TORCHDYNAMO_DISABLE=1 python tests/golden/make_golden.py <reference-root>

Writes ``tests/golden/golden.npz``.  Every array comes out of the reference's
own code (its CPU fallbacks for the Triton/CUDA ops, installed by
``lib/fast_kernels.py:install_cpu_fallbacks``):

* Hilbert codes of the four window orders and their permutations
  (``BK/base_models/order.py`` encoder, ``lib/fast_kernels.py:build_order_caches_fast``);
* the lexicographic permutation (``lib/fast_flow.py:_prepare_sample_geometry``);
* ``conv_indices`` (``lib/fast_kernels.py:build_conv_indices_fast``);
* RoPE tables (``precompute_rope_3d_table`` / ``precompute_rope_2d_cond``)
  and ``rope_nd`` at head_dim 128 (two pass-through channels);
* ``FlowModel.forward`` of small seeded models (cond, zero-context uncond),
  ``OptimizedLatDitRunner.forward_flow_fast(uncond=True)`` (1-token branch)
  and an exact Euler+CFG ``sample_fast`` run.

``BK/`` abbreviates ``baseline_repo/3dgen-main/``.  The weights of the small
models come from ``oracle.model.init_params`` (seeded), so the test side
rebuilds them instead of storing them.
"""
from __future__ import annotations

import importlib.util
import os
import sys
import types
from pathlib import Path

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
sys.dont_write_bytecode = True

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from oracle import model as om  # noqa: E402  (weights init shared with the tests)


def load_reference(ref: Path):
    for p in (ref, ref / "lib", ref / "baseline_repo" / "3dgen-main"):
        sys.path.insert(0, str(p))
    spec = importlib.util.spec_from_file_location("lib.fast_kernels", ref / "lib" / "fast_kernels.py")
    fk = importlib.util.module_from_spec(spec)
    sys.modules["lib.fast_kernels"] = fk
    spec.loader.exec_module(fk)
    fk.install_cpu_fallbacks()
    # stubs for packages the CPU path imports but never uses
    tm = types.ModuleType("trimesh")
    tm.Trimesh = object
    sys.modules.setdefault("trimesh", tm)
    d = types.ModuleType("diffusers")
    dc = types.ModuleType("diffusers.configuration_utils")

    class ConfigMixin:  # noqa: D401
        pass

    def register_to_config(fn):
        return fn

    dc.ConfigMixin = ConfigMixin
    dc.register_to_config = register_to_config
    dm = types.ModuleType("diffusers.models")
    dmm = types.ModuleType("diffusers.models.modeling_utils")
    dmm.ModelMixin = torch.nn.Module
    d.configuration_utils, d.models, dm.modeling_utils = dc, dm, dmm
    for name, mod in (("diffusers", d), ("diffusers.configuration_utils", dc),
                      ("diffusers.models", dm), ("diffusers.models.modeling_utils", dmm)):
        sys.modules.setdefault(name, mod)
    return fk


def seeded_voxels(n: int, grid: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    cells = rng.choice(grid ** 3, size=n, replace=False)
    return np.stack([cells // (grid * grid), (cells // grid) % grid, cells % grid], -1).astype(np.int32)


def shell_voxels(n: int, grid: int, radius: float, seed: int) -> np.ndarray:
    """A jittered one-voxel-thick sphere shell, subsampled to n voxels."""
    rng = np.random.default_rng(seed)
    m = 8 * n
    d = rng.normal(size=(m, 3))
    d /= np.linalg.norm(d, axis=1, keepdims=True)
    c = (grid - 1) / 2.0
    p = np.rint(c + radius * d + rng.normal(scale=0.3, size=(m, 3))).astype(np.int64)
    p = p[np.all((p >= 0) & (p < grid), axis=1)]
    p = np.unique(p, axis=0)
    p = p[rng.permutation(len(p))[:n]]
    return p.astype(np.int32)


def main(ref: Path) -> None:
    fk = load_reference(ref)
    import base_models.order as order
    import base_models.sparse as sp
    from models.generators.lat_dit import FlowModel

    out = {}

    # ---------------------------------------------------------------- geometry
    cases = {
        "g64": seeded_voxels(700, 64, 1),
        "g128": seeded_voxels(500, 128, 2),
        "shell": shell_voxels(600, 64, 24.0, 3),
        "edge": np.array([[0, 0, 0], [63, 63, 63], [0, 63, 0], [1, 0, 0], [0, 1, 0], [0, 0, 1],
                          [1, 1, 1], [62, 63, 63], [127, 0, 5], [2, 2, 2]], dtype=np.int32),
    }
    for name, vox in cases.items():
        out[f"{name}/vox"] = vox
        v = torch.from_numpy(vox)
        c_long = v.long()
        code = (c_long[:, 0] << 20) | (c_long[:, 1] << 10) | c_long[:, 2]
        perm = torch.argsort(code)                                  # fast_flow.py:675-679
        hc = torch.cat([torch.zeros(len(v), 1, dtype=torch.int32), v[perm]], 1).contiguous()
        out[f"{name}/perm"] = perm.numpy()
        out[f"{name}/h_coords"] = hc.numpy()
        codes = []
        for mode, conv in (("h", "xyz"), ("ht1", "yxz"), ("h1", "xyz"), ("ht", "yxz")):
            xyz = hc.clone()
            if mode.endswith("1"):
                xyz[:, 1:] += 1          # fused encoder shifts x,y,z only (fast_kernels.py:1146-1149)
            codes.append(order.encode_hilbert(xyz, conv))
        out[f"{name}/codes4"] = torch.stack(codes).numpy()
        caches = fk.build_order_caches_fast(hc, [len(hc)], ["h", "ht1", "h1", "ht"],
                                            {"patch_size": 64}, {}, torch.arange(len(hc)), use_triton=False)
        out[f"{name}/fwd4"] = torch.stack([c[0] for c in caches]).numpy()
        out[f"{name}/cu_seqlens"] = caches[0][2].numpy()
        out[f"{name}/conv_indices"] = fk.build_conv_indices_fast(hc, already_sorted=True)[0].numpy()
        out[f"{name}/conv_indices_unsorted"] = fk.build_conv_indices_fast(
            torch.cat([torch.zeros(len(v), 1, dtype=torch.int32), v], 1))[0].numpy()

    for res, hd in ((64, 96), (128, 128)):
        c, s = fk.precompute_rope_3d_table(res=res, base=128.0, head_dim=hd)
        out[f"rope3d_{res}_{hd}/cos"], out[f"rope3d_{res}_{hd}/sin"] = c.numpy(), s.numpy()
    for cs, hd in ((64, 96), (64, 128)):
        c, s = fk.precompute_rope_2d_cond(cond_size=cs, base=64.0, head_dim=hd)
        out[f"rope2d_{cs}_{hd}/cos"], out[f"rope2d_{cs}_{hd}/sin"] = c.numpy(), s.numpy()
    import models.generators.lat_dit as gld
    g = torch.Generator().manual_seed(5)
    xr = torch.randn(1, 40, 2, 128, generator=g)
    pr = torch.rand(1, 40, 3, generator=g) * 2 - 1
    out["rope_nd128/x"], out["rope_nd128/pos"] = xr.numpy(), pr.numpy()
    out["rope_nd128/out"] = gld.rope_nd(xr, pr, freq=128).numpy()

    # ---------------------------------------------------------------- model forward
    def run_model(tag, cfg: om.ModelConfig, n_vox, L, seed, t_val):
        p = om.init_params(cfg, seed, weight_std=0.05, bias_std=0.02, scale_jitter=0.1)
        flow = FlowModel(res=cfg.res, latent_dim=16, dim=cfg.dim, cond_depth=cfg.cond_depth, depth=cfg.depth,
                         head_dim=cfg.head_dim, rms=True, rope=True, pos_emb=False, ffn_conv=True,
                         ffn_rate=cfg.ffn_rate, patch=1, orders=list(cfg.orders), patch_size=cfg.patch_size)
        sd = {k[5:]: v for k, v in p.items() if k.startswith("flow.")}
        missing, unexpected = flow.load_state_dict(sd, strict=True), None
        flow.eval()
        vox = shell_voxels(n_vox, cfg.res, cfg.res * 0.36, seed + 100)
        gi = torch.Generator().manual_seed(seed + 7)
        xt = torch.randn(len(vox), 16, generator=gi)
        ctx = torch.randn(1, L, cfg.dim, generator=gi)
        coords = sp.sparse_coords([torch.from_numpy(vox)])
        t = torch.tensor([t_val * 1000.0])
        clf = torch.zeros(1, cfg.dim)
        with torch.no_grad():
            pos = flow(sp.SparseTensor(xt, coords.int()), t, clf, ctx).feats
            neg = flow(sp.SparseTensor(xt, coords.int()), t, clf, torch.zeros_like(ctx)).feats
        out[f"{tag}/vox"], out[f"{tag}/xt"], out[f"{tag}/ctx"] = vox, xt.numpy(), ctx[0].numpy()
        out[f"{tag}/pos"], out[f"{tag}/neg"] = pos.numpy(), neg.numpy()
        out[f"{tag}/meta"] = np.array([cfg.dim, cfg.head_dim, cfg.depth, cfg.cond_depth, cfg.res,
                                       cfg.patch_size, seed, L], dtype=np.int64)
        out[f"{tag}/t"] = np.array([t_val], dtype=np.float64)
        return p, flow, vox, xt, ctx

    cfg96 = om.ModelConfig(dim=192, head_dim=96, depth=3, cond_depth=1, res=64, patch_size=64)
    p96, flow96, vox96, xt96, ctx96 = run_model("m96", cfg96, 150, 41, 11, 0.75)
    cfg128 = om.ModelConfig(dim=256, head_dim=128, depth=2, cond_depth=1, res=64, patch_size=64)
    run_model("m128", cfg128, 130, 41, 12, 0.5)

    # ---------------------------------------------------------------- fast runner (1-token + sampler)
    try:
        from kandi3d_image23d.models.modeling_lat_dit import LatDitModel
        from lib.fast_flow import OptimizedLatDitRunner
        from lib.fast_sampler import SolverConfig
        from kandi3d_image23d.runtime import FlowMatchSamplingParams, LatDitConditioning

        mc = dict(res=64, latent_dim=16, dim=192, cond_depth=1, depth=3, head_dim=96, rms=True, rope=True,
                  pos_emb=False, ffn_conv=True, ffn_rate=2.5, patch=1, orders=["h", "ht1", "h1", "ht"],
                  patch_size=64, cfg=3.0, cfg_range=[0.5, 1.0], rescale_t=3.0)
        model = LatDitModel(dim=192, latent_dim=16, latent_scale=1.5, cond=["image_last"], model_config=mc)
        p = om.init_params(cfg96, 11, weight_std=0.05, bias_std=0.02, scale_jitter=0.1)
        sd = {k: v for k, v in p.items()}
        model.core.load_state_dict(sd, strict=True)
        model.eval()
        scfg = SolverConfig()
        for k, v in dict(solver_type="piecewise_euler", qaoa_enabled=False, cfg_stride=1,
                         cfg_cache_mode="exact", mid_block_cache_enabled=False, eval_cond_steps=[],
                         eval_uncond_steps=[], guidance_scale=3.0, num_inference_steps=4,
                         n_guided_steps=3, n_unguided_steps=1, cache_cond_block7_stride=1,
                         uncond_mid_block_cache=False, warmup_on_load=False).items():
            if hasattr(scfg, k):
                setattr(scfg, k, v)
        runner = OptimizedLatDitRunner(model, scfg)
        ctx_t = torch.from_numpy(out["m96/ctx"])[None]
        geom = runner._prepare_sample_geometry([torch.from_numpy(vox96)], ctx_t)
        xs = torch.from_numpy(out["m96/xt"])[geom["perm"]]
        with torch.no_grad():
            neg1 = runner.forward_flow_fast(xs, 0.75, ctx_t, torch.zeros(1, 192), geom, uncond=True)
            pos1 = runner.forward_flow_fast(xs, 0.75, ctx_t, torch.zeros(1, 192), geom, uncond=False)
        out["m96/neg_1tok_sorted"] = neg1.numpy()
        out["m96/pos_fast_sorted"] = pos1.numpy()
        # exact sampler through the runner: seeded DINO features and noise
        gi = torch.Generator().manual_seed(99)
        dino = torch.randn(1, 41, 1280, generator=gi)
        out["sample/dino"] = dino[0].numpy()
        gen = torch.Generator().manual_seed(1234)
        out["sample/noise"] = torch.randn(len(vox96), 16, generator=torch.Generator().manual_seed(1234)).numpy()
        with torch.no_grad():
            lat = runner.sample_fast([torch.from_numpy(vox96)], LatDitConditioning(dino_features=dino, batch_size=1),
                                     sampling=FlowMatchSamplingParams(guidance_scale=3.0, cfg_range=(0.5, 1.0),
                                                                      rescale_t=3.0, num_inference_steps=4),
                                     generator=gen)
        out["sample/latents"] = lat[0].numpy()
        out["sample/ok"] = np.array([1])
    except Exception as exc:  # the fixture records why the runner leg is missing
        print("runner leg skipped:", type(exc).__name__, exc)
        out["sample/ok"] = np.array([0])

    np.savez_compressed(HERE / "golden.npz", **out)
    print("wrote", HERE / "golden.npz", sum(v.nbytes for v in out.values()), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    main(Path(sys.argv[1]))
