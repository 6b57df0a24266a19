"""GPU parity at the full benchmark configurations.

* C1 one context block (dim 1536, 12 x 128, N = 4096, 4101 context tokens), both branches,
  against ``FlowModel.forward`` run by the reference on CPU in fp32 (``tests/golden/c1.npz``);
* C4 one NFE at full width and context (N = 16384, dim 1536, 4101 tokens) with 12 x 128 and
  16 x 96 heads on a depth-2 model, both branches (``c4nfe_*.npz``), and the full 24-block
  model through the exact 4-step sampler, 7 NFEs (``c4sample.npz``: the reference's own
  exact sampler on CPU, its unconditional NFEs on the full 4101-token zero context);
* C2 the QK-RMSNorm + RoPE3D + Hilbert-gather kernel at N = 16384, 65536 and 262144 uniform
  cells of 128^3 (Hilbert codes and orders bit-exact, q/k against fp32);
* C3 the dense 27-tap conv at N = 65536 (shell r = 56 in 128^3), 1536 -> 1536, on sampled
  output rows against the fp32 oracle.

The path computes in bf16 (fp32 accumulation and statistics), so every floating-point
comparison uses the bf16 bounds: relative L2 <= 1e-2 per NFE (and per kernel), <= 2e-2 on
the final latents.  The errors are printed (``pytest -rP``)."""
import numpy as np
import pytest
import torch

from vdit import _lib
from vdit import fast_kernels as fk
from vdit.fast_flow import OptimizedLatDitRunner
from vdit.fast_sampler import SolverConfig
from vdit.model import LatDitModel
from vdit.runtime import FlowMatchSamplingParams, LatDitConditioning
from vdit.workloads import shell_voxels, uniform_voxels

from oracle import geometry as geo
from oracle import model as om
from tests.golden import full_cases as fc

pytestmark = pytest.mark.gpu
DEV = "cuda"
NFE_TOL = 1e-2
LATENT_TOL = 2e-2


def rel(a, b):
    a = a.float().cpu() if torch.is_tensor(a) else torch.from_numpy(np.asarray(a)).float()
    b = b.float().cpu() if torch.is_tensor(b) else torch.from_numpy(np.asarray(b)).float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert _lib.device_error(clear=True) == 0


def _model(case: fc.Case, fx: dict):
    """The case's weights rebuilt on this host (checked against the fixture's checksum) and a
    runner on the GPU."""
    state = case.weights()
    want = float(fx["weight_checksum"][0])
    got = fc.weight_checksum(state)
    assert abs(got - want) <= 1e-9 * want, f"weights rebuilt differently on this host ({got!r} vs {want!r})"
    return OptimizedLatDitRunner(LatDitModel(case.arch(), state), SolverConfig(guidance_scale=3.0),
                                 device=torch.device(DEV))


def _check_inputs(fx: dict, tensors: dict):
    got = fc.checksums(tensors)
    assert np.allclose(got, fx["input_checksums"], rtol=1e-9, atol=0), "inputs rebuilt differently on this host"


@pytest.mark.parametrize("name", ["c1", "c4nfe_128", "c4nfe_96"])
def test_one_nfe_matches_reference_full_width(name):
    case, fx = fc.CASES[name], fc.load(name)
    vox = case.voxels()
    xt, ctx = case.nfe_inputs()
    _check_inputs(fx, {"vox": torch.from_numpy(vox), "xt": xt, "ctx": ctx})
    runner = _model(case, fx)
    ctx_d = ctx.to(DEV, torch.bfloat16)
    geom = runner._prepare_sample_geometry([torch.from_numpy(vox).to(DEV)], ctx_d)
    xs = xt.to(DEV)[geom["perm"]]
    up = geom["up_widx"]
    pos = runner.forward_flow_fast(xs, case.t, ctx_d, None, geom)[up]
    neg = runner.forward_flow_fast(xs, case.t, ctx_d, None, geom, uncond=True)[up]
    e_pos, e_neg = rel(pos, fx["pos"]), rel(neg, fx["neg"])
    print(f"\n{name}: rel L2 cond {e_pos:.3e}, 1-token uncond vs 4101-token zero context {e_neg:.3e}")
    assert e_pos <= NFE_TOL and e_neg <= NFE_TOL


def test_c4_sampler_matches_reference():
    """The full C4 model (24 blocks, 8 with context) through the exact sampler: 3 guided
    steps (conditional + exact 1-token NFE, CFG 3.0) and 1 unguided, against the reference's
    sampler on CPU."""
    case = fc.CASES["c4sample"]
    if not case.fixture_path().exists():
        pytest.skip("tests/golden/c4sample.npz not generated (make_golden_full.py c4sample)")
    fx = fc.load("c4sample")
    vox = case.voxels()
    dino, noise = case.sample_inputs()
    _check_inputs(fx, {"vox": torch.from_numpy(vox), "dino": dino, "noise": noise})
    runner = _model(case, fx)
    lat = runner.sample_fast([torch.from_numpy(vox).to(DEV)], LatDitConditioning(dino_features=dino.to(DEV)),
                             sampling=FlowMatchSamplingParams(guidance_scale=3.0, cfg_range=(0.5, 1.0), rescale_t=3.0,
                                                              num_inference_steps=4),
                             noise=noise.to(DEV))[0]
    err = rel(lat, fx["latents"])
    print(f"\nc4sample: final latents rel L2 {err:.3e}")
    assert lat.shape == (case.n, 16) and err <= LATENT_TOL


@pytest.mark.parametrize("n", [16384, 65536, 262144])
def test_c2_qknorm_rope3d_gather_sweep(n):
    heads, hd, res = 12, 128, 128
    vox = uniform_voxels(n, 128, 7000 + n)
    perm, _, hc = fk.lex_perm(torch.from_numpy(vox).to(DEV))
    p_o, _, hc_o = geo.lex_perm(vox)
    assert np.array_equal(perm.cpu().numpy(), p_o) and np.array_equal(hc.cpu().numpy(), hc_o)
    codes, fwd, _ = fk.hilbert4_orders(hc, 128, return_codes=True)
    codes_o = geo.encode_orders4(hc_o)
    assert np.array_equal(codes.cpu().numpy(), codes_o)
    fwd_o = np.stack([f for f, _ in geo.order_caches(codes_o)])
    assert np.array_equal(fwd.cpu().numpy(), fwd_o)
    g = torch.Generator(device=DEV).manual_seed(n)
    D = heads * hd
    qkv = torch.randn(n, 3 * D, device=DEV, generator=g).to(torch.bfloat16)
    qs = torch.ones(heads, hd, device=DEV)
    ks = torch.ones(heads, hd, device=DEV)
    cos, sin = fk.precompute_rope_3d_table(res, 128.0, hd, device=DEV)
    out = fk.fused_qknorm_rope3d_gather(qkv, qs, ks, cos, sin, hc, fwd[0], heads, hd).view(n, 3, heads, hd)
    # fp32 reference on (up to) 16384 output rows spread over the whole range
    rows = torch.from_numpy(np.unique(np.random.default_rng(n).integers(0, n, size=min(n, 16384))))
    src_rows = fwd[0].cpu()[rows]
    src = qkv.view(n, 3, heads, hd)[src_rows.to(DEV)].float().cpu()
    pos = (hc.float()[src_rows.to(DEV)][:, 1:].cpu() + 0.5) / res * 2 - 1
    q = om.rope_nd(om.rms_norm(src[:, 0]), pos, 128.0)
    k = om.rope_nd(om.rms_norm(src[:, 1]), pos, 128.0)
    got = out[rows.to(DEV)]
    e_q, e_k = rel(got[:, 0], q), rel(got[:, 1], k)
    print(f"\nC2 n={n}: rel L2 q {e_q:.3e}, k {e_k:.3e} ({len(rows)} rows)")
    assert e_q <= NFE_TOL and e_k <= NFE_TOL
    assert torch.equal(got[:, 2].cpu(), src[:, 2].to(torch.bfloat16))


def test_c3_dense_conv_sampled_rows():
    n, cin, cout = 65536, 1536, 1536
    vox = shell_voxels(n, 128, 56.0, 3)
    _, _, hc = fk.lex_perm(torch.from_numpy(vox).to(DEV))
    idx = fk.build_conv_indices_fast(hc, already_sorted=True)[0]
    assert np.array_equal(idx.cpu().numpy(), geo.conv_indices(hc.cpu().numpy()))
    g = torch.Generator(device=DEV).manual_seed(33)
    f = torch.randn(n, cin, device=DEV, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(27, cin, cout, device=DEV, generator=g)).to(torch.bfloat16)   # [27, Cin, Cout]
    b = 0.1 * torch.randn(cout, device=DEV, generator=g)
    out = fk.dense_sparse_conv3d(f, w.transpose(1, 2).contiguous(), b, [idx])
    # rows: a random spread, the first and last rows and the rows with the fewest / most taps
    taps = (idx >= 0).sum(1).cpu()
    rng = np.random.default_rng(34)
    rows = set(rng.choice(n, 384, replace=False).tolist()) | {0, n - 1}
    rows |= set(torch.argsort(taps)[:32].tolist()) | set(torch.argsort(taps)[-32:].tolist())
    rows = torch.tensor(sorted(rows))
    idx_c = idx.cpu()[rows]
    f_c, w_c = f.float().cpu(), w.float().cpu()
    ref = b.cpu().expand(len(rows), -1).clone()
    for d in range(27):
        sel = idx_c[:, d] >= 0
        if sel.any():
            ref[sel] += f_c[idx_c[sel, d].long()] @ w_c[d]
    e = rel(out[rows.to(DEV)], ref)
    print(f"\nC3 n={n} {cin}->{cout}: rel L2 {e:.3e} on {len(rows)} rows (taps per row {int(taps.min())}..{int(taps.max())})")
    assert e <= NFE_TOL
