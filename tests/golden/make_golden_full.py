"""Golden fixtures at the full benchmark configurations, by running the reference on CPU.

Usage (needs the reference checkout, read-only; no GPU; the sampler case takes tens of
minutes on a few host cores):

    TORCHDYNAMO_DISABLE=1 python tests/golden/make_golden_full.py <reference-root> c1 c4nfe_128 c4nfe_96 c4sample cfgreuse

Writes ``tests/golden/<case>.npz`` for each named case (``full_cases.CASES``):

* ``c1``, ``c4nfe_*``: ``FlowModel.forward`` (``BK/models/generators/lat_dit.py:743-824``)
  in fp32 with the context (``pos``) and with a zero context of the same length (``neg``),
  velocities in the input voxel order;
* ``c4sample``: the organiser baseline's exact sampler ``LatDitCore.sample_sparse``
  (``BK/kandi3d_image23d/modules/lat_dit/core.py:114-177``): Euler steps on the rescaled schedule
  t = [1, .9, .75, .5, 0], CFG 3.0 on the first three steps with the unconditional NFE run as
  ``FlowModel`` on a zero context of all 4101 tokens, then ``denormalize``; latents in the
  input order.  (The submission runner's ``sample_fast`` cannot run head_dim 128 on the CPU:
  its cached 3D RoPE, ``lib/fast_kernels.py:1040-1075``, needs head_dim % 6 == 0.  Its exact
  schedule is the same: ``lib/fast_sampler.py:670-732`` with cfg_range (0.5, 1) gives three
  guided steps, as the baseline's ``cfg_range[0] <= t`` test does with cfg_range (0.6, 1).)

``cfgreuse`` (-> ``cfg_reuse.npz``) pins the approximate CFG cache: the submission runner's
``sample_fast`` in its "neg_reuse" mode on the small model of ``golden.npz``.

Inputs and weights are rebuilt from seeds (``full_cases.py``), so only outputs and input
checksums are stored.  ``BK/`` abbreviates ``baseline_repo/3dgen-main/``.
"""
from __future__ import annotations

import os
import sys
import time
from pathlib import Path

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
sys.dont_write_bytecode = True

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from __graft_entry__ import load_package  # noqa: E402

load_package()

from tests.golden import full_cases as fc  # noqa: E402
from tests.golden.make_golden import load_reference  # noqa: E402


def flow_case(case: fc.Case) -> dict:
    import base_models.sparse as sp
    from models.generators.lat_dit import FlowModel

    state = case.weights()
    flow = FlowModel(res=case.grid, latent_dim=16, dim=case.dim, cond_depth=case.cond_depth, depth=case.depth,
                     head_dim=case.head_dim, rms=True, rope=True, pos_emb=False, ffn_conv=True, ffn_rate=2.5,
                     patch=1, orders=["h", "ht1", "h1", "ht"], patch_size=4096)
    flow.load_state_dict({k[5:]: v for k, v in state.items() if k.startswith("flow.")}, strict=True)
    flow.eval()
    vox = case.voxels()
    xt, ctx = case.nfe_inputs()
    coords = sp.sparse_coords([torch.from_numpy(vox)]).int()
    t = torch.tensor([case.t * 1000.0])
    clf = torch.zeros(1, case.dim)
    out = {}
    with torch.no_grad():
        t0 = time.time()
        out["pos"] = flow(sp.SparseTensor(xt, coords), t, clf, ctx[None]).feats.numpy()
        t1 = time.time()
        out["neg"] = flow(sp.SparseTensor(xt, coords), t, clf, torch.zeros_like(ctx)[None]).feats.numpy()
        t2 = time.time()
    print(f"{case.name}: pos {t1 - t0:.1f} s, neg {t2 - t1:.1f} s on {torch.get_num_threads()} threads")
    out["input_checksums"] = fc.checksums({"vox": torch.from_numpy(vox), "xt": xt, "ctx": ctx})
    out["weight_checksum"] = np.array([fc.weight_checksum(state)])
    return out


def sample_case(case: fc.Case) -> dict:
    from kandi3d_image23d.models.modeling_lat_dit import LatDitModel
    from kandi3d_image23d.runtime import FlowMatchSamplingParams, LatDitConditioning

    state = case.weights()
    wsum = fc.weight_checksum(state)
    mc = dict(case.model_config(), latent_dim=16, rms=True, rope=True, pos_emb=False, ffn_conv=True, patch=1,
              cfg=3.0, cfg_range=[0.6, 1.0], rescale_t=3.0)
    model = LatDitModel(dim=case.dim, latent_dim=16, latent_scale=1.5, cond=["image_last"], model_config=mc)
    model.core.load_state_dict(state, strict=True)
    del state
    model.eval()
    vox = case.voxels()
    dino, noise = case.sample_inputs()
    gen = torch.Generator().manual_seed(case.noise_seed)
    t0 = time.time()
    with torch.no_grad():
        lat = model.core.sample_sparse([torch.from_numpy(vox)], LatDitConditioning(dino_features=dino, batch_size=1),
                                       sampling=FlowMatchSamplingParams(guidance_scale=3.0, cfg_range=(0.6, 1.0),
                                                                        rescale_t=3.0, num_inference_steps=4),
                                       generator=gen)
    print(f"{case.name}: sample_sparse {time.time() - t0:.1f} s on {torch.get_num_threads()} threads")
    return {"latents": lat[0].numpy(),
            "input_checksums": fc.checksums({"vox": torch.from_numpy(vox), "dino": dino, "noise": noise}),
            "weight_checksum": np.array([wsum])}


def cfg_reuse_case() -> dict:
    """The submission runner's ``sample_fast`` (``lib/fast_flow.py:2523-3313``) with its approximate
    CFG cache on: ``cfg_cache_mode`` "neg_reuse", ``cfg_stride`` 2, ``eval_uncond_steps`` [0, 2]
    (its defaults, ``lib/fast_sampler.py:25-79``), QAOA and the context caches off, on the small
    head_dim-96 model and inputs of ``golden.npz`` (``m96``, ``sample/*``)."""
    from kandi3d_image23d.models.modeling_lat_dit import LatDitModel
    from kandi3d_image23d.runtime import FlowMatchSamplingParams, LatDitConditioning
    from lib.fast_flow import OptimizedLatDitRunner
    from lib.fast_sampler import SolverConfig
    from oracle import model as om

    golden = dict(np.load(HERE / "golden.npz"))
    cfg96 = om.ModelConfig(dim=192, head_dim=96, depth=3, cond_depth=1, res=64, patch_size=64)
    mc = dict(res=64, latent_dim=16, dim=192, cond_depth=1, depth=3, head_dim=96, rms=True, rope=True,
              pos_emb=False, ffn_conv=True, ffn_rate=2.5, patch=1, orders=["h", "ht1", "h1", "ht"],
              patch_size=64, cfg=3.0, cfg_range=[0.5, 1.0], rescale_t=3.0)
    model = LatDitModel(dim=192, latent_dim=16, latent_scale=1.5, cond=["image_last"], model_config=mc)
    model.core.load_state_dict(om.init_params(cfg96, 11, weight_std=0.05, bias_std=0.02, scale_jitter=0.1),
                               strict=True)
    model.eval()
    scfg = SolverConfig()
    for k, v in dict(solver_type="piecewise_euler", qaoa_enabled=False, cfg_stride=2, cfg_cache_mode="neg_reuse",
                     eval_uncond_steps=[0, 2], mid_block_cache_enabled=False, eval_cond_steps=[],
                     guidance_scale=3.0, num_inference_steps=4, n_guided_steps=3, n_unguided_steps=1,
                     cache_cond_block7_stride=1, uncond_mid_block_cache=False, warmup_on_load=False).items():
        if hasattr(scfg, k):
            setattr(scfg, k, v)
    runner = OptimizedLatDitRunner(model, scfg)
    dino = torch.from_numpy(golden["sample/dino"])[None]
    with torch.no_grad():
        lat = runner.sample_fast([torch.from_numpy(golden["m96/vox"])],
                                 LatDitConditioning(dino_features=dino, batch_size=1),
                                 sampling=FlowMatchSamplingParams(guidance_scale=3.0, cfg_range=(0.5, 1.0),
                                                                  rescale_t=3.0, num_inference_steps=4),
                                 generator=torch.Generator().manual_seed(1234))
    return {"latents": lat[0].numpy()}


def main(ref: Path, names) -> None:
    load_reference(ref)
    for name in names:
        if name == "cfgreuse":
            np.savez_compressed(HERE / "cfg_reuse.npz", **cfg_reuse_case())
            print("wrote", HERE / "cfg_reuse.npz")
            continue
        case = fc.CASES[name]
        out = sample_case(case) if name == "c4sample" else flow_case(case)
        out["meta"] = np.array([case.dim, case.head_dim, case.depth, case.cond_depth, case.n], dtype=np.int64)
        np.savez_compressed(case.fixture_path(), **out)
        print("wrote", case.fixture_path())


if __name__ == "__main__":
    if len(sys.argv) < 3:
        raise SystemExit(__doc__)
    main(Path(sys.argv[1]), sys.argv[2:])
