"""Pin the CPU oracle against fixtures produced by the reference itself
(``tests/golden/make_golden.py``): geometry bit-exact, model forward within
fp32 rounding."""
import numpy as np
import pytest
import torch

from oracle import geometry as geo
from oracle import model as om

CASES = ("g64", "g128", "shell", "edge")


@pytest.mark.parametrize("case", CASES)
def test_lex_perm(golden, case):
    perm, up, hc = geo.lex_perm(golden[f"{case}/vox"])
    assert np.array_equal(perm, golden[f"{case}/perm"])
    assert np.array_equal(hc, golden[f"{case}/h_coords"])
    assert np.array_equal(up[perm], np.arange(len(perm)))


@pytest.mark.parametrize("case", CASES)
def test_hilbert_codes_and_orders(golden, case):
    hc = golden[f"{case}/h_coords"]
    codes = geo.encode_orders4(hc)
    assert np.array_equal(codes, golden[f"{case}/codes4"])
    fwd = np.stack([f for f, _ in geo.order_caches(codes)])
    assert np.array_equal(fwd, golden[f"{case}/fwd4"])


@pytest.mark.parametrize("case", CASES)
def test_window_cu_seqlens(golden, case):
    n = len(golden[f"{case}/vox"])
    assert np.array_equal(geo.window_cu_seqlens(n, 64), golden[f"{case}/cu_seqlens"])


@pytest.mark.parametrize("case", CASES)
def test_conv_indices(golden, case):
    hc = golden[f"{case}/h_coords"]
    assert np.array_equal(geo.conv_indices(hc), golden[f"{case}/conv_indices"])
    vox = golden[f"{case}/vox"]
    raw = np.concatenate([np.zeros((len(vox), 1), np.int32), vox], 1)
    assert np.array_equal(geo.conv_indices(raw), golden[f"{case}/conv_indices_unsorted"])


@pytest.mark.parametrize("res,hd", [(64, 96), (128, 128)])
def test_rope3d_table(golden, res, hd):
    c, s = geo.rope3d_table(res, hd)
    assert np.array_equal(c, golden[f"rope3d_{res}_{hd}/cos"])
    assert np.array_equal(s, golden[f"rope3d_{res}_{hd}/sin"])


@pytest.mark.parametrize("hd", [96, 128])
def test_rope2d_table(golden, hd):
    c, s = geo.rope2d_table(64, hd)
    assert np.array_equal(c, golden[f"rope2d_64_{hd}/cos"].reshape(c.shape))
    assert np.array_equal(s, golden[f"rope2d_64_{hd}/sin"].reshape(s.shape))


def test_rope_nd_head128_passthrough(golden):
    x = torch.from_numpy(golden["rope_nd128/x"])
    pos = torch.from_numpy(golden["rope_nd128/pos"])
    out = om.rope_nd(x, pos, 128.0)
    ref = torch.from_numpy(golden["rope_nd128/out"])
    assert torch.allclose(out, ref, atol=1e-6, rtol=1e-6)
    assert torch.equal(out[..., 126:], x[..., 126:])


def _rel(a, b):
    return float(torch.linalg.norm(a - b) / torch.linalg.norm(b))


def _model(golden, tag):
    dim, hd, depth, cdepth, res, ps, seed, L = [int(v) for v in golden[f"{tag}/meta"]]
    cfg = om.ModelConfig(dim=dim, head_dim=hd, depth=depth, cond_depth=cdepth, res=res, patch_size=ps)
    p = om.init_params(cfg, seed, weight_std=0.05, bias_std=0.02, scale_jitter=0.1)
    geom = om.build_geometry(golden[f"{tag}/vox"], cfg)
    return cfg, p, geom


@pytest.mark.parametrize("tag", ["m96", "m128"])
def test_flow_forward_matches_reference(golden, tag):
    cfg, p, geom = _model(golden, tag)
    xt = torch.from_numpy(golden[f"{tag}/xt"])
    ctx = torch.from_numpy(golden[f"{tag}/ctx"])
    t = float(golden[f"{tag}/t"][0])
    pos = om.flow_forward(p, cfg, xt[geom.perm], t, ctx, geom)[geom.up_widx]
    neg = om.flow_forward(p, cfg, xt[geom.perm], t, torch.zeros_like(ctx), geom)[geom.up_widx]
    assert _rel(pos, torch.from_numpy(golden[f"{tag}/pos"])) < 1e-5
    assert _rel(neg, torch.from_numpy(golden[f"{tag}/neg"])) < 1e-5


def test_one_token_uncond_matches_reference(golden):
    cfg, p, geom = _model(golden, "m96")
    xt = torch.from_numpy(golden["m96/xt"])[geom.perm]
    neg1 = om.flow_forward_1tok(p, cfg, xt, float(golden["m96/t"][0]), geom)
    assert _rel(neg1, torch.from_numpy(golden["m96/neg_1tok_sorted"])) < 1e-5
    # and the exact condensation equals the full zero-context branch
    assert _rel(neg1[geom.up_widx], torch.from_numpy(golden["m96/neg"])) < 1e-5


def test_sampler_matches_reference(golden):
    if int(golden["sample/ok"][0]) != 1:
        pytest.skip("runner leg missing from fixtures")
    cfg, p, geom = _model(golden, "m96")
    dino = torch.from_numpy(golden["sample/dino"])
    ctx = torch.nn.functional.linear(dino, p["image_map.weight"], p["image_map.bias"])
    lat = om.sample(p, cfg, golden["m96/vox"], ctx, torch.from_numpy(golden["sample/noise"]),
                    guidance_scale=3.0, num_steps=4, n_guided=3)
    assert _rel(lat, torch.from_numpy(golden["sample/latents"])) < 1e-5


def test_cfg_reuse_sampler_matches_reference(golden):
    """The approximate CFG cache ("neg_reuse": the unconditional NFE at guided steps 0 and 2,
    reused with the CFG-Zero* projection, clean-endpoint blend and high-frequency boost at step
    1) against the reference runner's own ``sample_fast`` in that mode (``cfg_reuse.npz``)."""
    from pathlib import Path
    fx = np.load(Path(__file__).resolve().parent / "golden" / "cfg_reuse.npz")
    cfg, p, geom = _model(golden, "m96")
    dino = torch.from_numpy(golden["sample/dino"])
    ctx = torch.nn.functional.linear(dino, p["image_map.weight"], p["image_map.bias"])
    lat = om.sample(p, cfg, golden["m96/vox"], ctx, torch.from_numpy(golden["sample/noise"]),
                    guidance_scale=3.0, num_steps=4, n_guided=3, cfg_reuse={})
    assert _rel(lat, torch.from_numpy(fx["latents"])) < 1e-5


def test_schedule():
    t, guided = om.build_schedule(4, 3, 3.0, (0.5, 1.0))
    assert np.allclose(t.numpy(), [1.0, 0.9, 0.75, 0.5, 0.0], atol=1e-6)
    assert guided == [True, True, True, False]
