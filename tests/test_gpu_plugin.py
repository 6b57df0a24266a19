"""The plugin contract on the GPU, through ``Solution.generate`` (inherited from the
protocol class, never overridden): host-memory inputs as the harness passes them, a
batch of two samples, latents in the caller's voxel order, run metadata, the error
path; and run-twice determinism of the whole path (both NFE branches and the
sampler), as the reference's test plan asks of every kernel."""
import numpy as np
import pytest
import torch

from vdit.fast_sampler import SolverConfig
from vdit.model import LatDitModel
from vdit.runtime import LatDitConditioning
from vdit.solution import Solution

from oracle import model as om
from tests.golden.make_golden import shell_voxels

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / b.norm())


def small_solution(seed):
    cfg = om.ModelConfig(dim=256, head_dim=128, depth=2, cond_depth=1, res=64, patch_size=256)
    p = om.init_params(cfg, seed, weight_std=0.03, bias_std=0.02, scale_jitter=0.1)
    mc = {"dim": 256, "head_dim": 128, "depth": 2, "cond_depth": 1, "res": 64, "patch_size": 256,
          "latent_scale": cfg.latent_scale}
    sol = Solution(LatDitModel.from_state_dict(p, mc), SolverConfig(guidance_scale=3.0), device=DEV)
    return sol, p, cfg


def test_generate_contract_and_order():
    sol, p, cfg = small_solution(31)
    g = torch.Generator().manual_seed(32)
    voxs = [shell_voxels(500, 64, 20.0, 33), shell_voxels(310, 64, 17.0, 34)]
    dino = torch.randn(2, 5 + 64, 1280, generator=g).to(torch.float16)       # host memory, fp16
    cond = LatDitConditioning(dino_features=dino, batch_size=2)
    gen = torch.Generator(device=DEV).manual_seed(35)
    outs = sol.generate([torch.from_numpy(v) for v in voxs], conditioning=cond, generator=gen)
    assert len(outs) == 2
    for v, o in zip(voxs, outs):
        assert o.shape == (len(v), 16) and o.dtype == torch.float32 and bool(torch.isfinite(o).all())
    md = sol.last_run_metadata
    assert md["status"] == "ok" and md["elapsed_seconds"] > 0
    assert md["inputs"]["num_voxels"] == [len(v) for v in voxs] and md["inputs"]["batch_size"] == 2

    # the same noise draws through the CPU oracle: rows come back in the caller's voxel order
    g2 = torch.Generator(device=DEV).manual_seed(35)
    for i, (v, o) in enumerate(zip(voxs, outs)):
        noise = torch.randn(len(v), 16, device=DEV, generator=g2).cpu()
        ctx = torch.nn.functional.linear(dino[i].float(), p["image_map.weight"], p["image_map.bias"])
        ref = om.sample(p, cfg, v, ctx, noise, guidance_scale=3.0, num_steps=4, n_guided=3)
        assert rel(o, ref) < 2e-2


def test_generate_error_path_records_status():
    sol, _, _ = small_solution(41)
    bad = torch.zeros(10, 4, dtype=torch.int32)                           # coordinates must be [N, 3]
    cond = LatDitConditioning(dino_features=torch.zeros(1, 5 + 64, 1280, dtype=torch.float16))
    with pytest.raises(Exception):
        sol.generate([bad], conditioning=cond)
    assert sol.last_run_metadata["status"] == "error"
    assert sol.last_run_metadata["error_type"]


def test_runs_are_deterministic():
    sol, _, _ = small_solution(51)
    runner = sol.runner
    vox = torch.from_numpy(shell_voxels(700, 64, 22.0, 52)).to(DEV)
    g = torch.Generator().manual_seed(53)
    ctx = torch.randn(5 + 64, 256, generator=g).to(DEV, torch.bfloat16)
    xt = torch.randn(700, 16, generator=g).to(DEV)
    geom = runner._prepare_sample_geometry([vox], ctx)
    for uncond in (False, True):
        a = runner.forward_flow_fast(xt, 0.75, ctx, None, geom, uncond=uncond)
        b = runner.forward_flow_fast(xt, 0.75, ctx, None, geom, uncond=uncond)
        assert torch.equal(a, b), uncond
    dino = torch.randn(1, 5 + 64, 1280, generator=g).to(DEV)
    cond = LatDitConditioning(dino_features=dino)
    noise = torch.randn(700, 16, generator=g).to(DEV)
    s1 = runner.sample_fast([vox], cond, noise=noise)[0]
    s2 = runner.sample_fast([vox], cond, noise=noise)[0]
    assert torch.equal(s1, s2)


def test_generate_from_sample_cache(tmp_path):
    """The on-disk sample format into the plugin: vox_idxi.npz + 4view_000_dinov3.npz (fp16
    features mapped by image_map on the GPU), latents in the file's voxel order."""
    from vdit import ingest
    sol, p, cfg = small_solution(71)
    d = tmp_path / "s0" / "cache"
    d.mkdir(parents=True)
    vox = shell_voxels(400, 64, 18.0, 72)
    np.savez(d / "vox_idxi.npz", vox_idxi=vox)
    g = np.random.default_rng(73)
    np.savez(d / "4view_000_dinov3.npz", feats=g.standard_normal((1, 5 + 64, 1280)).astype(np.float16),
             token=g.standard_normal((1, 1280)).astype(np.float16))
    vl, cond = ingest.load_sample(tmp_path / "s0", pin_memory=True)
    gen = torch.Generator(device=DEV).manual_seed(74)
    out = sol.generate(vl, conditioning=cond, generator=gen)[0]
    assert out.shape == (400, 16) and bool(torch.isfinite(out).all())
    g2 = torch.Generator(device=DEV).manual_seed(74)
    noise = torch.randn(400, 16, device=DEV, generator=g2).cpu()
    ctx = torch.nn.functional.linear(cond.dino_features[0].float(), p["image_map.weight"], p["image_map.bias"])
    ref = om.sample(p, cfg, vox, ctx, noise, guidance_scale=3.0, num_steps=4, n_guided=3)
    assert rel(out, ref) < 2e-2
