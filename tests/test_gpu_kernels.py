"""GPU parity of each kernel through the C ABI: integer geometry bit-exact
against the oracle / reference fixtures, floating-point kernels against fp32
references (tolerances in each test)."""
import math

import numpy as np
import pytest
import torch

from vdit import _lib
from vdit import fast_kernels as fk

from oracle import geometry as geo
from oracle import model as om

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def unique_cells(n, grid, seed):
    rng = np.random.default_rng(seed)
    c = rng.choice(grid ** 3, size=n, replace=False)
    return np.stack([c // (grid * grid), (c // grid) % grid, c % grid], -1).astype(np.int32)


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert _lib.device_error(clear=True) == 0


# ----------------------------------------------------------------------------- geometry (bit-exact)

@pytest.mark.parametrize("case", ["g64", "g128", "shell", "edge"])
def test_geometry_matches_reference_fixtures(golden, case):
    vox = torch.from_numpy(golden[f"{case}/vox"]).to(DEV)
    perm, up, hc = fk.lex_perm(vox)
    assert np.array_equal(perm.cpu().numpy(), golden[f"{case}/perm"])
    assert np.array_equal(hc.cpu().numpy(), golden[f"{case}/h_coords"])
    assert torch.equal(up[perm].cpu(), torch.arange(len(vox)))
    for bound in (128, 1024):
        codes, fwd, bwd = fk.hilbert4_orders(hc, bound, return_codes=True)
        assert np.array_equal(codes.cpu().numpy(), golden[f"{case}/codes4"])
        assert np.array_equal(fwd.cpu().numpy(), golden[f"{case}/fwd4"])
        for i in range(4):
            assert torch.equal(bwd[i][fwd[i]].cpu(), torch.arange(len(vox)))
    idx = fk.build_conv_indices_fast(hc, already_sorted=True)[0]
    assert np.array_equal(idx.cpu().numpy(), golden[f"{case}/conv_indices"])
    raw = torch.cat([torch.zeros(len(vox), 1, dtype=torch.int32, device=DEV), vox], 1)
    idx2 = fk.build_conv_indices_fast(raw)[0]
    assert np.array_equal(idx2.cpu().numpy(), golden[f"{case}/conv_indices_unsorted"])


@pytest.mark.parametrize("n", [1, 2, 3, 5, 127, 4097, 262144])
def test_geometry_sizes_128grid(n):
    """C2 geometry: unique uniform voxels in 128^3 (21-bit codes), up to 262144."""
    vox = unique_cells(n, 128, n)
    g = geo.sample_geometry(vox)
    perm, up, hc = fk.lex_perm(torch.from_numpy(vox).to(DEV))
    assert np.array_equal(perm.cpu().numpy(), g["perm"])
    codes, fwd, _ = fk.hilbert4_orders(hc, 128, return_codes=True)
    assert np.array_equal(codes.cpu().numpy(), g["codes4"])
    assert np.array_equal(fwd.cpu().numpy(), np.stack([f for f, _ in g["order_caches"]]))
    if n <= 5000:
        idx = fk.build_conv_indices_fast(hc, already_sorted=True)[0]
        assert np.array_equal(idx.cpu().numpy(), g["conv_indices"])
    assert int(codes.max()) < 2 ** 24


def test_conv_indices_dense_shell():
    from tests.golden.make_golden import shell_voxels
    vox = shell_voxels(16384, 64, 30.0, 7)
    g = geo.sample_geometry(vox)
    _, _, hc = fk.lex_perm(torch.from_numpy(vox).to(DEV))
    idx = fk.build_conv_indices_fast(hc, already_sorted=True)[0].cpu().numpy()
    assert np.array_equal(idx, g["conv_indices"])
    assert (idx >= 0).sum(1).mean() > 3     # a surface: several neighbours per voxel


@pytest.mark.parametrize("res,hd", [(64, 96), (128, 128)])
def test_rope_tables(golden, res, hd):
    c, s = fk.precompute_rope_3d_table(res, 128.0, hd, device=DEV)
    np.testing.assert_array_max_ulp(c.cpu().numpy(), golden[f"rope3d_{res}_{hd}/cos"], maxulp=1)
    np.testing.assert_array_max_ulp(s.cpu().numpy(), golden[f"rope3d_{res}_{hd}/sin"], maxulp=1)
    c2, s2 = fk.precompute_rope_2d_cond(64, 64.0, hd, device=DEV)
    np.testing.assert_array_max_ulp(c2.cpu().numpy().reshape(-1), golden[f"rope2d_64_{hd}/cos"].reshape(-1), maxulp=1)
    np.testing.assert_array_max_ulp(s2.cpu().numpy().reshape(-1), golden[f"rope2d_64_{hd}/sin"].reshape(-1), maxulp=1)


# ----------------------------------------------------------------------------- row kernels

@pytest.mark.parametrize("m,d", [(1, 1536), (1000, 1536), (333, 192), (4101, 768)])
def test_modulate_and_gate_add(m, d):
    g = torch.Generator(device=DEV).manual_seed(m + d)
    x = torch.randn(m, d, device=DEV, generator=g).to(torch.bfloat16)
    h = torch.randn(m, d, device=DEV, generator=g).to(torch.bfloat16)
    s1, sh, gt = [torch.randn(d, device=DEV, generator=g) * 0.3 + o for o in (1.0, 0.0, 0.0)]
    ref = om.layer_norm(x.float()) * s1 + sh
    assert rel(fk.fast_modulate(x, None, s1, sh), ref) < 1e-2        # bf16 output rounding
    x2 = x.clone()
    mod = fk.fast_gate_add_and_modulate(x2, h, gt, s1, sh)
    xr = x.float() + h.float() * gt
    assert rel(x2, xr) < 5e-3
    assert rel(mod, om.layer_norm(x2.float()) * s1 + sh) < 1e-2
    x3 = x.clone()
    fk.fast_gate_add_and_modulate(x3, h[0], gt, None, None, broadcast_h=True)
    assert rel(x3, x.float() + h[0].float() * gt) < 5e-3


@pytest.mark.parametrize("m,d", [(700, 1536), (5000, 1536), (4096, 768)])
def test_gate_add2_matches_two_passes(m, d):
    """Two gated residuals in one pass (the second a broadcast row) against two gate-add
    passes: the same bits, then the same modulation."""
    g = torch.Generator(device=DEV).manual_seed(m + 3)
    x = torch.randn(m, d, device=DEV, generator=g).to(torch.bfloat16)
    h = torch.randn(m, d, device=DEV, generator=g).to(torch.bfloat16)
    c = torch.randn(d, device=DEV, generator=g).to(torch.bfloat16)
    g1, g2, s1, sh = [torch.randn(d, device=DEV, generator=g) * 0.3 + o for o in (0.0, 0.0, 1.0, 0.0)]
    xa = x.clone()
    ma = fk.fast_gate_add2_and_modulate(xa, h, g1, c, g2, s1, sh)
    xb = x.clone()
    fk.fast_gate_add_and_modulate(xb, h, g1, None, None)
    mb = fk.fast_gate_add_and_modulate(xb, c, g2, s1, sh, broadcast_h=True)
    assert torch.equal(xa, xb) and torch.equal(ma, mb)


@pytest.mark.parametrize("m,d,stride_h", [(4096, 1536, False), (9001, 1536, True), (5000, 768, False)])
def test_gate_add_staged_matches_rowwise(m, d, stride_h):
    """m >= 4096 rows take the persistent staged kernel; chunks below that the
    one-row-per-warp kernel.  Both must produce identical bits."""
    g = torch.Generator(device=DEV).manual_seed(m)
    x = torch.randn(m, d, device=DEV, generator=g).to(torch.bfloat16)
    hs = torch.randn(m, 2 * d if stride_h else d, device=DEV, generator=g).to(torch.bfloat16)
    h = hs[:, d:] if stride_h else hs                   # a row stride of 2d
    s1, sh, gt = [torch.randn(d, device=DEV, generator=g) * 0.3 + o for o in (1.0, 0.0, 0.0)]
    xa = x.clone()
    mod_a = fk.fast_gate_add_and_modulate(xa, h, gt, s1, sh)
    xb = x.clone()
    mods = [fk.fast_gate_add_and_modulate(xb[i:i + 2048], h[i:i + 2048], gt, s1, sh) for i in range(0, m, 2048)]
    assert torch.equal(xa, xb) and torch.equal(mod_a, torch.cat(mods))
    xc = x.clone()
    fk.fast_gate_add_and_modulate(xc, h, gt, None, None)
    assert torch.equal(xc, xa)
    # plain modulation: the staged kernel without its gate-add against the row-per-warp kernel
    mod_s = fk.fast_modulate(x, None, s1, sh)
    mod_r = torch.cat([fk.fast_modulate(x[i:i + 2048], None, s1, sh) for i in range(0, m, 2048)])
    assert torch.equal(mod_s, mod_r)


@pytest.mark.parametrize("m,d", [(777, 1536), (1, 1536), (16384, 1536), (301, 1000), (64, 2048)])
def test_out_modulate_unpatchify(m, d):
    """Ragged 128-row tiles (m % 128), a ragged last 64-column chunk (d = 1000), one row."""
    g = torch.Generator(device=DEV).manual_seed(3 + m + d)
    x = torch.randn(m, d, device=DEV, generator=g).to(torch.bfloat16)
    s1 = 1 + 0.1 * torch.randn(d, device=DEV, generator=g)
    sh = 0.1 * torch.randn(d, device=DEV, generator=g)
    w = 0.05 * torch.randn(16, d, device=DEV, generator=g)
    out = fk.fast_out_modulate_unpatchify(x, None, s1, sh, w)
    mod = (om.layer_norm(x.float()) * s1 + sh).to(torch.bfloat16).float()   # rounded as the reference does
    ref = mod @ w.t()
    # fp32 accuracy from the three-part bf16 split of the weight (bf16 weights alone: ~2e-3)
    assert out.dtype == torch.float32 and out.shape == (m, 16) and rel(out, ref) < 5e-5
    for r in (0, m - 1):                                                    # each row on its own
        assert rel(out[r], ref[r]) < 1e-4


def test_split_weight3_is_exact():
    """hi + mid + lo reproduces every fp32 weight (three bf16 parts carry the 24-bit significand)."""
    g = torch.Generator(device=DEV).manual_seed(11)
    w = torch.randn(16, 1536, device=DEV, generator=g) * torch.logspace(-4, 2, 1536, device=DEV)
    w3 = fk.split_weight3(w)
    assert w3.dtype == torch.bfloat16 and w3.shape == (48, 1536)
    parts = w3.double().reshape(3, 16, 1536)
    assert torch.equal(parts.sum(0), w.double())
    assert torch.equal(w3[:16], w.to(torch.bfloat16))                    # hi = bf16(w)


@pytest.mark.parametrize("m,d", [(777, 1536), (1, 1536), (16384, 1536), (301, 1000), (64, 2048), (130, 8)])
def test_unpatchify_project(m, d):
    """The projection alone on modulated rows: ragged row tiles (m % 128), a ragged last column
    chunk (d % 64), fp32-accurate against a float64 product (bf16 weights would miss by ~2e-3)."""
    g = torch.Generator(device=DEV).manual_seed(5 + m + d)
    x = torch.randn(m, d, device=DEV, generator=g).to(torch.bfloat16)
    s1 = 1 + 0.1 * torch.randn(d, device=DEV, generator=g)
    sh = 0.1 * torch.randn(d, device=DEV, generator=g)
    w = 0.05 * torch.randn(16, d, device=DEV, generator=g)
    y = fk.fast_modulate(x, None, s1, sh)
    out = fk.unpatchify_project(y, fk.split_weight3(w))
    ref = y.double() @ w.double().t()
    assert out.dtype == torch.float32 and out.shape == (m, 16) and rel(out, ref) < 5e-5
    fused = fk.fast_out_modulate_unpatchify(x, None, s1, sh, w)           # the one-call fused form
    assert rel(out, fused) < 5e-5


@pytest.mark.parametrize("n,d", [(500, 1536), (16384, 1536), (1, 64), (1025, 200)])
def test_patchify(n, d):
    """Ragged row tiles (n % 512) and a channel tile with idle lanes (d = 200)."""
    g = torch.Generator(device=DEV).manual_seed(4 + n)
    xt = torch.randn(n, 16, device=DEV, generator=g)
    w = torch.randn(d, 16, device=DEV, generator=g) * 0.2
    out = fk.patchify(xt, w)
    ref = (xt.double() @ w.double().t()).float()
    assert out.shape == (n, d) and rel(out, ref) < 5e-3
    assert (out.float() - ref).abs().max() <= 2 ** -7 * ref.abs().max() + 1e-6   # bf16 rounding only


@pytest.mark.parametrize("heads,hd,res", [(12, 128, 128), (16, 96, 64), (2, 96, 64)])
def test_qknorm_rope3d_gather(heads, hd, res):
    n = 3000
    vox = unique_cells(n, res, hd)
    _, _, hc = fk.lex_perm(torch.from_numpy(vox).to(DEV))
    g = torch.Generator(device=DEV).manual_seed(heads)
    D = heads * hd
    qkv = torch.randn(n, 3 * D, device=DEV, generator=g).to(torch.bfloat16)
    qs = 1 + 0.1 * torch.randn(heads, hd, device=DEV, generator=g)
    ks = 1 + 0.1 * torch.randn(heads, hd, device=DEV, generator=g)
    fwd = torch.randperm(n, device=DEV)
    cos, sin = fk.precompute_rope_3d_table(res, 128.0, hd, device=DEV)
    out = fk.fused_qknorm_rope3d_gather(qkv, qs, ks, cos, sin, hc, fwd, heads, hd).view(n, 3, heads, hd)
    src = qkv.float()[fwd].view(n, 3, heads, hd).cpu()
    pos = ((hc.float()[fwd][:, 1:] + 0.5) / res * 2 - 1).cpu()
    q = om.rope_nd(om.rms_norm(src[:, 0]) * qs.cpu(), pos, 128.0)
    k = om.rope_nd(om.rms_norm(src[:, 1]) * ks.cpu(), pos, 128.0)
    assert rel(out[:, 0], q) < 1e-2 and rel(out[:, 1], k) < 1e-2
    assert torch.equal(out[:, 2], qkv.view(n, 3, heads, hd)[fwd][:, 2])


@pytest.mark.parametrize("heads,hd", [(12, 128), (16, 96)])
def test_qknorm_rope2d(heads, hd):
    L = 4101
    g = torch.Generator(device=DEV).manual_seed(hd)
    D = heads * hd
    qkv = torch.randn(L, 3 * D, device=DEV, generator=g).to(torch.bfloat16)
    ref_in = qkv.float().view(L, 3, heads, hd).cpu()
    qs = 1 + 0.1 * torch.randn(heads, hd, device=DEV, generator=g)
    ks = 1 + 0.1 * torch.randn(heads, hd, device=DEV, generator=g)
    cos, sin = fk.precompute_rope_2d_cond(64, 64.0, hd, device=DEV)
    fk.fused_qknorm_rope2d_cond_inplace(qkv, qs, ks, cos, sin, heads, hd)
    out = qkv.view(L, 3, heads, hd)
    cpos = om.cond_positions(L)
    q = om.rms_norm(ref_in[:, 0]) * qs.cpu()
    k = om.rms_norm(ref_in[:, 1]) * ks.cpu()
    q = torch.cat([q[:5], om.rope_nd(q[5:], cpos, 64.0)])
    k = torch.cat([k[:5], om.rope_nd(k[5:], cpos, 64.0)])
    assert rel(out[:, 0], q) < 1e-2 and rel(out[:, 1], k) < 1e-2
    assert torch.equal(out[:, 2].float().cpu(), ref_in[:, 2])


def test_swiglu():
    g = torch.Generator(device=DEV).manual_seed(9)
    h = torch.randn(4101, 7680, device=DEV, generator=g).to(torch.bfloat16)
    a, gg = h.float().chunk(2, -1)
    assert rel(fk.fast_swiglu_from_packed(h), torch.nn.functional.silu(gg) * a) < 1e-2


@pytest.mark.parametrize("c", [7680, 960])
def test_dwconv27(c):
    from tests.golden.make_golden import shell_voxels
    vox = shell_voxels(6000, 64, 24.0, 11)
    _, _, hc = fk.lex_perm(torch.from_numpy(vox).to(DEV))
    idx = fk.build_conv_indices_fast(hc, already_sorted=True)[0]
    g = torch.Generator(device=DEV).manual_seed(c)
    n = len(vox)
    h = torch.randn(n, c, device=DEV, generator=g).to(torch.bfloat16)
    w = 0.2 * torch.randn(27, c, device=DEV, generator=g)
    b = 0.1 * torch.randn(c, device=DEV, generator=g)
    ref = om.dwconv27(h.float().cpu(), w.cpu(), b.cpu(), idx.cpu())
    assert rel(fk.fast_sparse_conv3d(h, w, b, [idx]), ref) < 1e-2
    a, gg = ref.chunk(2, -1)
    assert rel(fk.fast_sparse_conv3d(h, w, b, [idx], fuse_swiglu=True), torch.nn.functional.silu(gg) * a) < 1e-2


def _planned_case(vox, c, seed):
    _, _, hc = fk.lex_perm(torch.from_numpy(vox).to(DEV))
    idx = fk.build_conv_indices_fast(hc, already_sorted=True)[0]
    fwd, _ = fk.hilbert4_orders(hc, 1024)
    g = torch.Generator(device=DEV).manual_seed(seed)
    n = hc.shape[0]
    h = torch.randn(n, c, device=DEV, generator=g).to(torch.bfloat16)
    w = 0.2 * torch.randn(27, c, device=DEV, generator=g)
    b = 0.1 * torch.randn(c, device=DEV, generator=g)
    return h, w, b, idx, fwd


@pytest.mark.parametrize("case", ["shell", "shell_ragged", "scattered", "cube", "tiny"])
def test_dwconv27_swiglu_planned(case):
    """The staged kernel equals the gather kernel bit for bit: staged blocks on a
    surface, scattered voxels, a dense cube, a partial last block and a single
    voxel; in lexicographic order most blocks of the shell and the cube exceed
    the slot capacity and run from global memory."""
    from tests.golden.make_golden import shell_voxels
    if case == "shell":
        vox, c = shell_voxels(16384, 64, 36.0, 0), 7680
    elif case == "shell_ragged":
        vox, c = shell_voxels(5001, 64, 24.0, 3), 1024
    elif case == "scattered":
        rng = np.random.default_rng(5)
        vox, c = np.unique(rng.integers(0, 64, size=(3000, 3)), axis=0).astype(np.int32), 512
    elif case == "cube":
        g = np.meshgrid(np.arange(20), np.arange(20), np.arange(20), indexing="ij")
        vox, c = np.stack(g, -1).reshape(-1, 3).astype(np.int32), 256
    else:
        vox, c = np.array([[3, 4, 5]], np.int32), 256
    h, w, b, idx, fwd = _planned_case(vox, c, 17)
    ref = fk.fast_sparse_conv3d(h, w, b, [idx], fuse_swiglu=True)
    perm = _pair_interleave(c)
    hp, wp, bp = h[:, perm].contiguous(), w[:, perm].contiguous(), b[perm].contiguous()
    for k in (0, 2):
        plan = fk.build_conv_plan([idx], fwd[k])
        out = fk.fast_sparse_conv3d_swiglu_planned(hp, wp, bp, plan)
        assert torch.equal(out, ref), (case, k, (out.float() - ref.float()).abs().max().item())
    # identity order: lexicographic blocks, mostly global-memory on the shell
    plan = fk.build_conv_plan([idx], torch.arange(h.shape[0], device=DEV))
    assert torch.equal(fk.fast_sparse_conv3d_swiglu_planned(hp, wp, bp, plan), ref)


@pytest.mark.parametrize("case", ["shell", "cube", "tiny"])
def test_dwconv27_swiglu_planned_bf16_weights(case):
    """With bf16-valued weights (a bf16 model upcast to fp32) the bf16-operand FMAs give
    the bits of the fp32-weight path: staged blocks (shell), blocks computed from global
    memory (the dense cube in lexicographic order) and a single voxel."""
    from tests.golden.make_golden import shell_voxels
    if case == "shell":
        vox, c = shell_voxels(16384, 64, 36.0, 0), 7680
    elif case == "cube":
        g = np.meshgrid(np.arange(20), np.arange(20), np.arange(20), indexing="ij")
        vox, c = np.stack(g, -1).reshape(-1, 3).astype(np.int32), 256
    else:
        vox, c = np.array([[3, 4, 5]], np.int32), 256
    h, w, b, idx, fwd = _planned_case(vox, c, 23)
    w = w.to(torch.bfloat16).float()
    assert fk.weights_are_bf16(w) and not fk.weights_are_bf16(w + 1e-3)
    perm = _pair_interleave(c)
    hp, wp, bp = h[:, perm].contiguous(), w[:, perm].contiguous(), b[perm].contiguous()
    for order in (fwd[0], torch.arange(h.shape[0], device=DEV)):
        plan = fk.build_conv_plan([idx], order)
        ref = fk.fast_sparse_conv3d_swiglu_planned(hp, wp, bp, plan)
        out = fk.fast_sparse_conv3d_swiglu_planned(hp, wp, bp, plan, bf16_weights=True)
        assert torch.equal(out, ref), (case, (out.float() - ref.float()).abs().max().item())


def _pair_interleave(c):
    """Column order (a[2k], a[2k+1], gate[2k], gate[2k+1]) of the staged conv's input."""
    return torch.arange(c, device=DEV).view(2, c // 4, 2).permute(1, 0, 2).reshape(-1)


def test_dwconv27_planned_vs_oracle():
    from tests.golden.make_golden import shell_voxels
    h, w, b, idx, fwd = _planned_case(shell_voxels(3000, 64, 20.0, 2), 768, 4)
    ref = om.dwconv27(h.float().cpu(), w.cpu(), b.cpu(), idx.cpu())
    a, gg = ref.chunk(2, -1)
    plan = fk.build_conv_plan([idx], fwd[0])
    perm = _pair_interleave(768)
    out = fk.fast_sparse_conv3d_swiglu_planned(h[:, perm].contiguous(), w[:, perm].contiguous(),
                                               b[perm].contiguous(), plan)
    assert rel(out, torch.nn.functional.silu(gg) * a) < 1e-2


# ----------------------------------------------------------------------------- attention

def ref_attention(q, k, v, cu_q, cu_k, heads, hd):
    out = torch.empty(q.shape[0], heads, hd, device=q.device)
    qf, kf, vf = (t.float().reshape(t.shape[0], heads, hd) for t in (q, k, v))
    for i in range(len(cu_q) - 1):
        a, b, c, d = cu_q[i], cu_q[i + 1], cu_k[i], cu_k[i + 1]
        if b > a:
            out[a:b] = torch.nn.functional.scaled_dot_product_attention(
                qf[a:b].transpose(0, 1), kf[c:d].transpose(0, 1), vf[c:d].transpose(0, 1)).transpose(0, 1)
    return out.reshape(q.shape[0], heads * hd)


@pytest.mark.parametrize("heads,hd", [(12, 128), (16, 96)])
@pytest.mark.parametrize("cu_q,cu_k", [
    ([0, 4096, 5000], [0, 4096, 5000]),          # windows, ragged tail
    ([0, 1000], [0, 4101]),                      # voxel -> context
    ([0, 4101], [0, 1000]),                      # context -> voxel
    ([0, 1], [0, 1]), ([0, 130], [0, 3]), ([0, 7, 300, 301], [0, 129, 130, 700]),
])
def test_attention_matches_fp32(heads, hd, cu_q, cu_k):
    g = torch.Generator(device=DEV).manual_seed(len(cu_q) * 7 + cu_q[-1] + hd)
    D = heads * hd
    nq, nk = cu_q[-1], cu_k[-1]
    q = torch.randn(nq, D, device=DEV, generator=g).to(torch.bfloat16)
    kv = torch.randn(nk, 2 * D, device=DEV, generator=g).to(torch.bfloat16)   # packed, strided views
    out = fk.attention(q, kv[:, :D], kv[:, D:], cu_q, cu_k, heads, hd)
    ref = ref_attention(q, kv[:, :D], kv[:, D:], cu_q, cu_k, heads, hd)
    assert rel(out, ref) < 1e-2


@pytest.mark.parametrize("heads,hd", [(12, 128), (16, 96)])
def test_attention_empty_key_segment_gives_zeros(heads, hd):
    """A segment with queries and no keys writes zero rows; the segments around it are unaffected
    (a query tile of the empty segment shares no barrier with them)."""
    cu_q, cu_k = [0, 130, 330, 331], [0, 0, 257, 600]
    g = torch.Generator(device=DEV).manual_seed(91 + hd)
    D = heads * hd
    q = torch.randn(cu_q[-1], D, device=DEV, generator=g).to(torch.bfloat16)
    kv = torch.randn(cu_k[-1], 2 * D, device=DEV, generator=g).to(torch.bfloat16)
    out = fk.attention(q, kv[:, :D], kv[:, D:], cu_q, cu_k, heads, hd)
    assert torch.count_nonzero(out[:130]) == 0
    ref = ref_attention(q[130:], kv[:, :D], kv[:, D:], [0, 200, 201], [0, 257, 600], heads, hd)
    assert rel(out[130:], ref) < 1e-2


def test_attention_scatter_and_large_logits():
    heads, hd, n = 12, 128, 4096 + 700
    g = torch.Generator(device=DEV).manual_seed(1)
    qkv = torch.randn(n, 3 * heads * hd, device=DEV, generator=g)
    qkv[:, : heads * hd] *= 6.0          # peaky softmax: exercises the deferred O rescale
    qkv = qkv.to(torch.bfloat16)
    D = heads * hd
    rows = torch.randperm(n, device=DEV)
    out = fk.flash_varlen_qkvpacked_already_sorted(qkv, torch.tensor([0, 4096, n]), 4096, heads, hd,
                                                   out_rows=rows)
    ref = ref_attention(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], [0, 4096, n], [0, 4096, n], heads, hd)
    assert rel(out[rows], ref) < 1e-2


def test_attention_late_dominant_keys():
    """Keys in later tiles whose scores exceed every earlier score by hundreds (in log2
    units): the running max jumps far past what the deferred rescale absorbs."""
    heads, hd, n = 4, 128, 4096
    g = torch.Generator(device=DEV).manual_seed(2)
    qkv = torch.randn(n, 3 * heads * hd, device=DEV, generator=g)
    D = heads * hd
    qkv[:, :D] *= 6.0
    for r in (1000, 2500, 4000):                              # keys in tiles 7, 19 and 31
        qkv[r, D:2 * D] *= 40.0
    qkv = qkv.to(torch.bfloat16)
    out = fk.flash_varlen_qkvpacked_already_sorted(qkv, torch.tensor([0, n]), n, heads, hd)
    ref = ref_attention(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], [0, n], [0, n], heads, hd)
    assert bool(torch.isfinite(out.float()).all())
    assert rel(out, ref) < 1e-2


@pytest.mark.parametrize("n,heads,hd", [(1, 12, 128), (1000, 12, 128), (16384, 12, 128), (5000, 16, 96)])
def test_attention_1q(n, heads, hd):
    g = torch.Generator(device=DEV).manual_seed(n)
    D = heads * hd
    q = torch.randn(D, device=DEV, generator=g)
    kv = torch.randn(n, 2 * D, device=DEV, generator=g).to(torch.bfloat16)
    out = fk.attention_1q(q, kv, heads, hd)
    ref = ref_attention(q.to(torch.bfloat16)[None], kv[:, :D], kv[:, D:], [0, 1], [0, n], heads, hd)[0]
    assert rel(out, ref) < 1e-2


# ----------------------------------------------------------------------------- dense 27-tap conv

@pytest.mark.parametrize("n,cin,cout", [(700, 64, 256), (3000, 128, 512), (4096, 1536, 256)])
def test_dense_conv27(n, cin, cout):
    from tests.golden.make_golden import shell_voxels
    vox = shell_voxels(n, 64, 24.0, cin)
    _, _, hc = fk.lex_perm(torch.from_numpy(vox).to(DEV))
    idx = fk.build_conv_indices_fast(hc, already_sorted=True)[0]
    g = torch.Generator(device=DEV).manual_seed(n + cin)
    f = torch.randn(n, cin, device=DEV, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(3, 3, 3, cin, cout, device=DEV, generator=g)).to(torch.bfloat16).float()
    b = 0.1 * torch.randn(cout, device=DEV, generator=g)
    wt = w.reshape(27, cin, cout).transpose(1, 2).contiguous().to(torch.bfloat16)   # [27, cout, cin]
    out = fk.dense_sparse_conv3d(f, wt, b, [idx])
    ref = om.dense_conv27(f.float().cpu(), w.cpu(), b.cpu(), idx.cpu())
    assert rel(out, ref) < 1e-2


def test_dense_conv27_rejects_bad_shapes():
    f = torch.zeros(10, 100, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="unsupported"):
        fk.dense_sparse_conv3d(f, torch.zeros(27, 256, 100, device=DEV, dtype=torch.bfloat16),
                               torch.zeros(256, device=DEV), [torch.zeros(10, 27, dtype=torch.int32, device=DEV)])


# ----------------------------------------------------------------------------- block linears (tcgen05 GEMM)

@pytest.mark.parametrize("m,k,n,bias,strided", [(1, 64, 256, True, False), (300, 1536, 512, True, False),
                                                 (4101, 1536, 4608, True, False), (16384, 1536, 1536, False, False),
                                                 (1000, 3840, 1536, True, True), (129, 128, 768, True, True),
                                                 (16384, 1536, 1536, True, True), (4101, 1536, 7680, True, False),
                                                 (5000, 256, 576, True, False), (2000, 512, 640, False, True),
                                                 (300, 480, 960, True, False), (4101, 200, 320, True, True),
                                                 (777, 72, 200, True, True), (1, 1536, 1536, True, False)])
def test_linear_matches_fp32(m, k, n, bias, strided):
    """Pair tiles of 256, 192 or 128 columns, the widest that divides n (n = 576 takes
    192-column tiles, n = 640 128-column tiles with the 8-stage ring); a partial last
    k-step (k = 480, 72, 200) and a partial last column tile (n = 320, 200) read zeros."""
    g = torch.Generator(device=DEV).manual_seed(m + k + n)
    a_full = torch.randn(m, k + (64 if strided else 0), device=DEV, generator=g).to(torch.bfloat16)
    a = a_full[:, 16:16 + k] if strided else a_full             # row stride k + 64, 32-byte offset
    w = (0.03 * torch.randn(n, k, device=DEV, generator=g)).to(torch.bfloat16)
    b = (0.1 * torch.randn(n, device=DEV, generator=g)).to(torch.bfloat16) if bias else None
    out_full = torch.full((m, n + (256 if strided else 0)), 7.0, device=DEV, dtype=torch.bfloat16)
    out = out_full[:, :n]
    fk.linear(a, w, b, out=out)
    ref = a.float() @ w.float().t() + (b.float() if bias else 0.0)
    assert rel(out, ref) < 5e-3                                  # bf16 output rounding
    if strided:
        assert bool((out_full[:, n:] == 7.0).all())              # columns past n untouched
    cub = torch.nn.functional.linear(a, w, b)
    assert rel(out, cub) < 5e-3


def test_linear_rejects_bad_shapes():
    a = torch.zeros(10, 100, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="unsupported"):            # k not a multiple of 8
        fk.linear(a, torch.zeros(256, 100, device=DEV, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="unsupported"):            # n not a multiple of 8
        fk.linear(torch.zeros(10, 128, device=DEV, dtype=torch.bfloat16),
                  torch.zeros(100, 128, device=DEV, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="unsupported"):
        fk.linear(torch.zeros(10, 128, device=DEV, dtype=torch.bfloat16),
                  torch.zeros(324, 128, device=DEV, dtype=torch.bfloat16))


# ----------------------------------------------------------------------------- one-row linears (GEMV)

def _ln_mod_ref(x, s1, sh):
    mu = x.mean()
    var = ((x - mu) ** 2).mean()
    return ((x - mu) * torch.rsqrt(var + 1e-6) * s1 + sh).to(torch.bfloat16).float()


@pytest.mark.parametrize("mode,wdt,n,k,batch,silu_out", [
    (fk.GEMV_X_BF16, torch.bfloat16, 1536, 1536, 1, False),
    (fk.GEMV_X_BF16, torch.bfloat16, 3072, 1536, 1, False),
    (fk.GEMV_X_LN_MOD, torch.bfloat16, 3072, 1536, 1, False),
    (fk.GEMV_X_LN_MOD, torch.bfloat16, 1536, 1536, 16, False),
    (fk.GEMV_X_SWIGLU, torch.bfloat16, 1536, 3840, 1, False),
    (fk.GEMV_X_F32, torch.float32, 6144, 256, 1, True),
    (fk.GEMV_X_F32, torch.float32, 1536, 6144, 1, True),
    (fk.GEMV_X_F32, torch.float32, 24 * 9 * 256, 256, 1, False),
    (fk.GEMV_X_BF16, torch.bfloat16, 40, 104, 3, False),
    (fk.GEMV_X_F32, torch.float32, 7, 12, 1, False),
])
def test_gemv_matches_fp32(mode, wdt, n, k, batch, silu_out):
    """Every prologue (plain bf16 / fp32 vector, LayerNorm-modulated fp32 vector with
    per-entry scale and shift, SwiGLU of a packed bf16 vector), bf16 and fp32 weights,
    batches, short rows (k = 12, 104: fewer chunks than lanes)."""
    g = torch.Generator(device=DEV).manual_seed(n + k + batch)
    w = (0.03 * torch.randn(batch, n, k, device=DEV, generator=g)).to(wdt)
    b = (0.1 * torch.randn(batch, n, device=DEV, generator=g)).to(wdt)
    s1 = 1 + 0.2 * torch.randn(batch, 2, k, device=DEV, generator=g)
    if mode == fk.GEMV_X_SWIGLU:
        x = torch.randn(2 * k, device=DEV, generator=g).to(torch.bfloat16)
        xr = (torch.nn.functional.silu(x[k:].float()) * x[:k].float()).to(torch.bfloat16).float()
    elif mode == fk.GEMV_X_BF16:
        x = torch.randn(k, device=DEV, generator=g).to(torch.bfloat16)
        xr = x.float()
    else:
        x = 3 + torch.randn(k, device=DEV, generator=g)
        xr = x
    xs = [xr] * batch
    if mode == fk.GEMV_X_LN_MOD:
        xs = [_ln_mod_ref(x, s1[i, 0], s1[i, 1]) for i in range(batch)]
    ww = w if batch > 1 else w[0]
    bb = b if batch > 1 else b[0]
    kw = dict(x_mode=mode, out_dtype=torch.float32 if wdt == torch.float32 else torch.bfloat16, silu_out=silu_out)
    if mode == fk.GEMV_X_LN_MOD:
        kw.update(mod_scale=s1[:, 0] if batch > 1 else s1[0, 0], mod_shift=s1[:, 1] if batch > 1 else s1[0, 1])
    out = fk.gemv(x, ww, bb, **kw)
    ref = torch.stack([w[i].float() @ xs[i] + b[i].float() for i in range(batch)])
    if silu_out:
        ref = torch.nn.functional.silu(ref)
    out = out.reshape(batch, n)
    tol = 1e-5 if wdt == torch.float32 else 5e-3                  # fp32 / bf16 output rounding
    assert rel(out, ref) < tol


def test_gemv_rejects_bad_arguments():
    w = torch.zeros(64, 1536, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        fk.gemv(torch.zeros(1500, device=DEV, dtype=torch.bfloat16), w)
    with pytest.raises(ValueError):
        fk.gemv(torch.zeros(1536, device=DEV), w, x_mode=fk.GEMV_X_LN_MOD)
    with pytest.raises(RuntimeError, match="unsupported"):
        fk.gemv(torch.zeros(9000, device=DEV, dtype=torch.bfloat16),
                torch.zeros(8, 9000, device=DEV, dtype=torch.bfloat16))


@pytest.mark.parametrize("n,heads,hd,res", [(3000, 12, 128, 128), (16384, 12, 128, 64), (300, 2, 128, 64),
                                             (3000, 16, 96, 64), (5000, 2, 96, 128)])
def test_linear_qkv_rope3d_matches_two_pass(n, heads, hd, res):
    """The fused epilogue against the two-pass path (GEMM, then the QK-norm / RoPE /
    gather kernel) and the fp32 oracle; rows land at bwd[r]."""
    K = 1536
    vox = unique_cells(n, res, n + heads)
    _, _, hc = fk.lex_perm(torch.from_numpy(vox).to(DEV))
    g = torch.Generator(device=DEV).manual_seed(n + res)
    D = heads * hd
    a = torch.randn(n, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (0.03 * torch.randn(3 * D, K, device=DEV, generator=g)).to(torch.bfloat16)
    b = (0.1 * torch.randn(3 * D, device=DEV, generator=g)).to(torch.bfloat16)
    qs = 1 + 0.1 * torch.randn(D, device=DEV, generator=g)
    ks = 1 + 0.1 * torch.randn(D, device=DEV, generator=g)
    fwd = torch.randperm(n, device=DEV, generator=g)
    bwd = torch.empty_like(fwd)
    bwd[fwd] = torch.arange(n, device=DEV)
    cos, sin = fk.precompute_rope_3d_table(res, 128.0, hd, device=DEV)
    fused = fk.linear_qkv_rope3d(a, w, b, qs, ks, cos, sin, hc, bwd, heads, hd)
    two = fk.fused_qknorm_rope3d_gather(torch.nn.functional.linear(a, w, b), qs, ks, cos, sin, hc, fwd, heads, hd)
    d = (fused.float() - two.float()).abs()
    # same bf16 GEMM output; only the order of the RMS sum differs (a rare 1-ulp bf16 flip)
    assert float((d > 0).float().mean()) < 1e-3 and float(d.max()) <= 0.0625
    assert torch.equal(fused[:, 2 * D:], two[:, 2 * D:])          # v rows: the bf16 GEMM output, moved
    src = (a.float() @ w.float().t() + b.float())[fwd].view(n, 3, heads, hd).cpu()
    pos = ((hc.float()[fwd][:, 1:] + 0.5) / res * 2 - 1).cpu()
    q = om.rope_nd(om.rms_norm(src[:, 0]) * qs.view(heads, hd).cpu(), pos, 128.0)
    fv = fused.view(n, 3, heads, hd)
    assert rel(fv[:, 0], q) < 1e-2


def test_linear_qkv_rope3d_rejects_odd_shapes():
    n, K = 64, 128
    a = torch.zeros(n, K, device=DEV, dtype=torch.bfloat16)
    hc = torch.zeros(n, 4, device=DEV, dtype=torch.int32)
    bwd = torch.arange(n, device=DEV)
    cos, sin = fk.precompute_rope_3d_table(64, 128.0, 128, device=DEV)
    for heads, hd in ((3, 128), (3, 96), (2, 64)):                 # odd head counts; head_dim 64
        D = heads * hd
        with pytest.raises(RuntimeError, match="unsupported"):
            fk.linear_qkv_rope3d(a, torch.zeros(3 * D, K, device=DEV, dtype=torch.bfloat16),
                                 torch.zeros(3 * D, device=DEV, dtype=torch.bfloat16), torch.ones(D, device=DEV),
                                 torch.ones(D, device=DEV), cos, sin, hc, bwd, heads, hd)


@pytest.mark.parametrize("n,heads,hd", [(16384, 12, 128), (1, 12, 128), (777, 16, 96), (5000, 2, 128)])
def test_attention_1q_wide(n, heads, hd):
    """The single query over K/V = x W^T + b without forming K/V, against forming them
    (F.linear, the bf16 K/V the reference attends over) with the single-query kernel,
    and against fp32 math."""
    g = torch.Generator(device=DEV).manual_seed(n + heads)
    D = heads * hd
    x = torch.randn(n, D, device=DEV, generator=g).to(torch.bfloat16)
    w_kv = (0.04 * torch.randn(2 * D, D, device=DEV, generator=g)).to(torch.bfloat16)
    b_kv = (0.3 * torch.randn(2 * D, device=DEV, generator=g)).to(torch.bfloat16)
    q = (2.0 * torch.randn(D, device=DEV, generator=g)).to(torch.bfloat16)
    out = fk.attention_1q_wide(q, x, w_kv, b_kv, heads, hd)
    kv = torch.nn.functional.linear(x, w_kv, b_kv)
    two = fk.attention_1q(q, kv, heads, hd)
    kf = (x.float() @ w_kv[:D].float().t() + b_kv[:D].float()).view(n, heads, hd)
    vf = (x.float() @ w_kv[D:].float().t() + b_kv[D:].float()).view(n, heads, hd)
    p = torch.softmax(torch.einsum("hd,nhd->hn", q.float().view(heads, hd), kf) / math.sqrt(hd), dim=1)
    ref = torch.einsum("hn,nhd->hd", p, vf).reshape(-1)
    assert rel(out, ref) < 1e-2
    assert rel(out, two) < 2e-2
