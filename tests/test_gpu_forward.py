"""GPU parity of the whole path against the CPU oracle: one NFE (cond branch,
exact 1-token uncond branch) and the 4-step exact sampler.  Tolerances:
per-NFE relative L2 <= 1e-2 (bf16), final latents <= 2e-2."""
import numpy as np
import pytest
import torch

from vdit import _lib
from vdit import fast_kernels as fk
from vdit.fast_flow import OptimizedLatDitRunner
from vdit.fast_sampler import SolverConfig
from vdit.model import LatDitModel
from vdit.runtime import LatDitConditioning

from oracle import model as om
from tests.golden.make_golden import shell_voxels

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / b.norm())


def build(dim, hd, depth, cdepth, n, side, patch, seed):
    cfg = om.ModelConfig(dim=dim, head_dim=hd, depth=depth, cond_depth=cdepth, res=64, patch_size=patch)
    p = om.init_params(cfg, seed, weight_std=0.03, bias_std=0.02, scale_jitter=0.1)
    mc = {"dim": dim, "head_dim": hd, "depth": depth, "cond_depth": cdepth, "res": 64, "patch_size": patch,
          "latent_scale": cfg.latent_scale}
    runner = OptimizedLatDitRunner(LatDitModel.from_state_dict(p, mc), SolverConfig(guidance_scale=3.0),
                                   device=torch.device(DEV))
    vox = shell_voxels(n, 64, 22.0, seed)
    L = 5 + side * side
    g = torch.Generator().manual_seed(seed + 1)
    ctx = torch.randn(L, dim, generator=g)
    xt = torch.randn(len(vox), 16, generator=g)
    return cfg, p, runner, vox, ctx, xt


@pytest.mark.parametrize("dim,hd", [(768, 128), (768, 96)])
def test_one_nfe_matches_oracle(dim, hd):
    cfg, p, runner, vox, ctx, xt = build(dim, hd, depth=3, cdepth=2, n=900, side=16, patch=256, seed=dim + hd)
    geom_o = om.build_geometry(vox, cfg)
    xs = xt[geom_o.perm]
    t = 0.75
    pos_o = om.flow_forward(p, cfg, xs, t, ctx, geom_o)
    neg_o = om.flow_forward_1tok(p, cfg, xs, t, geom_o)
    neg_full_o = om.flow_forward(p, cfg, xs, t, torch.zeros_like(ctx), geom_o)
    assert rel(neg_o, neg_full_o) < 1e-5        # the oracle's own exactness check
    ctx_d = ctx.to(DEV, torch.bfloat16)
    geom = runner._prepare_sample_geometry([torch.from_numpy(vox).to(DEV)], ctx_d)
    assert torch.equal(geom["perm"].cpu(), geom_o.perm)
    xs_d = xs.to(DEV)
    pos = runner.forward_flow_fast(xs_d, t, ctx_d, None, geom)
    neg = runner.forward_flow_fast(xs_d, t, ctx_d, None, geom, uncond=True)
    assert rel(pos, pos_o) < 1e-2
    assert rel(neg, neg_o) < 1e-2
    # block-0 sharing off gives the same uncond result
    runner.solver_config.ditfastattn_b0_msa_share = False
    neg2 = runner.forward_flow_fast(xs_d, t, ctx_d, None, geom, uncond=True)
    assert rel(neg2, neg) < 1e-3
    assert _lib.device_error() == 0


def test_bf16_conv_weights_take_the_bf16_operand_conv():
    """A model whose conv weights hold bf16 values (a bf16 checkpoint upcast, as the reference
    does) runs the bf16-operand conv in every block, with the same bits as the fp32-weight
    conv, in both branches."""
    cfg = om.ModelConfig(dim=512, head_dim=128, depth=2, cond_depth=1, res=64, patch_size=256)
    p = om.init_params(cfg, 5, weight_std=0.03, bias_std=0.02, scale_jitter=0.1)
    keys = [k for k in p if k.endswith("ffn_conv.weight")]
    assert len(keys) == cfg.depth
    for k in keys:
        p[k] = p[k].to(torch.bfloat16).float()
    mc = {"dim": 512, "head_dim": 128, "depth": 2, "cond_depth": 1, "res": 64, "patch_size": 256,
          "latent_scale": cfg.latent_scale}
    runner = OptimizedLatDitRunner(LatDitModel.from_state_dict(p, mc), SolverConfig(guidance_scale=3.0),
                                   device=torch.device(DEV))
    assert runner.ffn_interleaved and runner.conv_bf16w == [True, True]
    vox = shell_voxels(600, 64, 20.0, 9)
    g = torch.Generator().manual_seed(10)
    ctx = torch.randn(5 + 64, 512, generator=g).to(DEV, torch.bfloat16)
    geom = runner._prepare_sample_geometry([torch.from_numpy(vox).to(DEV)], ctx)
    xs = torch.randn(len(vox), 16, generator=g).to(DEV)
    out = [runner.forward_flow_fast(xs, 0.5, ctx, None, geom, uncond=u) for u in (False, True)]
    runner.conv_bf16w = [False, False]
    ref = [runner.forward_flow_fast(xs, 0.5, ctx, None, geom, uncond=u) for u in (False, True)]
    for a, b in zip(out, ref):
        assert torch.equal(a, b)
    assert _lib.device_error() == 0


def test_sampler_matches_oracle():
    cfg, p, runner, vox, ctx_unused, _ = build(512, 128, depth=2, cdepth=1, n=700, side=8, patch=256, seed=5)
    g = torch.Generator().manual_seed(6)
    dino = torch.randn(1, 5 + 64, 1280, generator=g)
    noise = torch.randn(len(vox), 16, generator=g)
    ctx = torch.nn.functional.linear(dino[0], p["image_map.weight"], p["image_map.bias"])
    lat_o = om.sample(p, cfg, vox, ctx, noise, guidance_scale=3.0, num_steps=4, n_guided=3)
    lat = runner.sample_fast([torch.from_numpy(vox).to(DEV)], LatDitConditioning(dino_features=dino.to(DEV)),
                             noise=noise.to(DEV))[0]
    assert lat.shape == (len(vox), 16) and lat.dtype == torch.float32
    assert rel(lat, lat_o) < 2e-2
    assert _lib.device_error() == 0


@pytest.mark.parametrize("zero_star,blend,hf,with_x0", [(True, 0.08, 0.02, True), (True, 0.08, 0.0, False),
                                                       (False, 0.08, 0.02, True)])
def test_cfg_reuse_step_matches_oracle(zero_star, blend, hf, with_x0):
    """One Euler step of the approximate CFG cache (reuse of the last unconditional velocity)
    against the oracle's restatement of the reference's formulas, fp32."""
    n = 5000
    g = torch.Generator().manual_seed(21)
    xt, vp, ln, x0 = (torch.randn(n, 16, generator=g) for _ in range(4))
    t_eval, dt, gs = 0.75, 0.25, 3.0
    delta = om.cfg_reuse_delta(vp, ln, xt, x0 if with_x0 else None, t_eval, zero_star=zero_star,
                               endpoint_blend=blend, hf_boost=hf / max(1e-9, 1.0 - t_eval) if hf else 0.0)
    want = xt - dt * (vp + gs * delta)
    got = xt.to(DEV).contiguous()
    fk.cfg_reuse_euler_(got, vp.to(DEV), ln.to(DEV), x0.to(DEV) if with_x0 else None, gs, dt, t_eval, blend, hf,
                        zero_star)
    assert rel(got, want) < 1e-5
    assert _lib.device_error() == 0


def test_sampler_cfg_reuse_matches_reference(golden):
    """The approximate sampler (unconditional NFE at guided steps 0 and 2, reused at step 1)
    against the reference runner's ``sample_fast`` in its "neg_reuse" mode, on the small
    head_dim-96 model of the golden fixtures (``tests/golden/cfg_reuse.npz``)."""
    from pathlib import Path
    fx = np.load(Path(__file__).resolve().parent / "golden" / "cfg_reuse.npz")
    cfg = om.ModelConfig(dim=192, head_dim=96, depth=3, cond_depth=1, res=64, patch_size=64)
    p = om.init_params(cfg, 11, weight_std=0.05, bias_std=0.02, scale_jitter=0.1)
    mc = {"dim": 192, "head_dim": 96, "depth": 3, "cond_depth": 1, "res": 64, "patch_size": 64,
          "latent_scale": cfg.latent_scale}
    solver = SolverConfig(guidance_scale=3.0).enable_approximate_cfg_cache()
    runner = OptimizedLatDitRunner(LatDitModel.from_state_dict(p, mc), solver, device=torch.device(DEV))
    dino = torch.from_numpy(golden["sample/dino"])[None]
    lat = runner.sample_fast([torch.from_numpy(golden["m96/vox"]).to(DEV)],
                             LatDitConditioning(dino_features=dino.to(DEV)),
                             noise=torch.from_numpy(golden["sample/noise"]).to(DEV))[0]
    err = rel(lat, torch.from_numpy(fx["latents"]))
    print(f"\ncfg reuse sampler: rel L2 vs the reference's approximate sampler {err:.3e}")
    assert err < 2e-2
    assert _lib.device_error() == 0


def test_graph_replay_matches_eager():
    """The CUDA-graph sampler equals the eager one on the sample it was captured with
    and on another sample of the same size (new voxels, context and noise copied in)."""
    cfg, p, runner, vox, ctx_unused, _ = build(512, 128, depth=2, cdepth=1, n=700, side=8, patch=256, seed=7)
    g = torch.Generator().manual_seed(8)
    cases = []
    for seed in (11, 12):
        v = shell_voxels(700, 64, 22.0, seed)
        assert len(v) == 700
        dino = torch.randn(1, 5 + 64, 1280, generator=g).to(DEV)
        cases.append((torch.from_numpy(v).to(DEV), LatDitConditioning(dino_features=dino),
                      torch.randn(700, 16, generator=g).to(DEV)))
    for v, cond, noise in cases:
        eager = runner.sample_fast([v], cond, noise=noise)[0]
        runner.cuda_graph = True
        graphed = runner.sample_fast([v], cond, noise=noise)[0]
        runner.cuda_graph = False
        assert rel(graphed, eager) < 1e-4
    assert len(runner._graphs) == 1
    assert _lib.device_error() == 0


def test_one_nfe_large_n_matches_oracle():
    """N = 32768 voxels of an ellipsoid-shell union in 128^3 (eight 4096-voxel windows,
    the production window size, the staged conv over 256 blocks): one NFE of each branch."""
    from vdit.workloads import ellipsoid_union
    dim, hd = 256, 128
    cfg = om.ModelConfig(dim=dim, head_dim=hd, depth=2, cond_depth=1, res=128, patch_size=4096)
    p = om.init_params(cfg, 21, weight_std=0.03, bias_std=0.02, scale_jitter=0.1)
    mc = {"dim": dim, "head_dim": hd, "depth": 2, "cond_depth": 1, "res": 128, "patch_size": 4096,
          "latent_scale": cfg.latent_scale}
    runner = OptimizedLatDitRunner(LatDitModel.from_state_dict(p, mc), SolverConfig(guidance_scale=3.0),
                                   device=torch.device(DEV))
    vox = ellipsoid_union(32768, 128, 3)
    assert len(vox) == 32768
    g = torch.Generator().manual_seed(22)
    ctx = torch.randn(5 + 64, dim, generator=g)
    xt = torch.randn(len(vox), 16, generator=g)
    geom_o = om.build_geometry(vox, cfg)
    xs = xt[geom_o.perm]
    t = 0.9
    pos_o = om.flow_forward(p, cfg, xs, t, ctx, geom_o)
    neg_o = om.flow_forward_1tok(p, cfg, xs, t, geom_o)
    ctx_d = ctx.to(DEV, torch.bfloat16)
    geom = runner._prepare_sample_geometry([torch.from_numpy(vox).to(DEV)], ctx_d)
    assert torch.equal(geom["perm"].cpu(), geom_o.perm)
    xs_d = xs.to(DEV)
    assert rel(runner.forward_flow_fast(xs_d, t, ctx_d, None, geom), pos_o) < 1e-2
    assert rel(runner.forward_flow_fast(xs_d, t, ctx_d, None, geom, uncond=True), neg_o) < 1e-2
    assert _lib.device_error() == 0
