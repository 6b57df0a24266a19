"""Our kernels against the reference's own CUDA kernels (BK/ops/libsparse/conv.cu, built
unmodified into oracle/_ref by oracle/build_ref.py) on the same inputs: conv_indices
bit-exact, the depthwise 27-tap conv bit-exact, the dense 27-tap conv within bf16
tolerance.  Each case also prints both kernels' times (CUDA events) for the reference-
kernel comparison.  Skipped where the checker library was not built (no reference
checkout in the build container)."""
import numpy as np
import pytest
import torch

from vdit import fast_kernels as fk

from oracle.build_ref import load_built
from tests.golden.make_golden import shell_voxels

pytestmark = pytest.mark.gpu
DEV = "cuda"
REF = load_built()
needs_ref = pytest.mark.skipif(REF is None, reason="oracle/_ref was not built (no reference checkout)")


def _time(fn, reps=10):
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def _geometry(n, grid, r, seed):
    vox = torch.from_numpy(shell_voxels(n, grid, r, seed)).to(DEV)
    _, _, hc = fk.lex_perm(vox)
    idx = fk.build_conv_indices_fast(hc, already_sorted=True)[0]
    ref_idx = REF.conv_indices(hc.contiguous())
    return hc, idx, ref_idx


@needs_ref
@pytest.mark.parametrize("n,grid,r", [(16384, 64, 36.0), (4097, 64, 24.0), (65536, 128, 56.0)])
def test_conv_indices_matches_reference_kernel(n, grid, r):
    hc, idx, ref_idx = _geometry(n, grid, r, n)
    assert ref_idx[0].shape[0] == (n + 3) // 4 * 4                   # the reference pads to 4 rows
    assert torch.equal(idx, ref_idx[0][:n])
    t_ours = _time(lambda: fk.build_conv_indices_fast(hc, already_sorted=True))
    t_ref = _time(lambda: REF.conv_indices(hc))
    print(f"\nconv_indices n={n}: ours {t_ours * 1e3:.1f} us, reference {t_ref * 1e3:.1f} us")


@needs_ref
@pytest.mark.parametrize("n,c", [(16384, 7680), (3001, 256)])
def test_depthwise_conv_matches_reference_kernel(n, c):
    """fast_sparse_conv3d (gather form, the reference's layout) against conv_fwd, and the
    staged form with fused SwiGLU against SwiGLU of conv_fwd's output."""
    hc, idx, ref_idx = _geometry(n, 64, 36.0, c)
    g = torch.Generator(device=DEV).manual_seed(n)
    h = torch.randn(n, c, device=DEV, generator=g).to(torch.bfloat16)
    w = 0.2 * torch.randn(3, 3, 3, c, device=DEV, generator=g)
    b = 0.1 * torch.randn(c, device=DEV, generator=g)
    ref = REF.conv_fwd(h, w.contiguous(), b, ref_idx)
    ours = fk.fast_sparse_conv3d(h, w, b, [idx])
    assert torch.equal(ours, ref)
    t_ours = _time(lambda: fk.fast_sparse_conv3d(h, w, b, [idx]))
    t_ref = _time(lambda: REF.conv_fwd(h, w, b, ref_idx))
    print(f"\nconv_fwd (depthwise) n={n} c={c}: ours {t_ours * 1e3:.1f} us, reference {t_ref * 1e3:.1f} us")


@needs_ref
def test_dense_conv_matches_reference_kernel():
    """dense_sparse_conv3d (tcgen05, bf16) against the reference's dense_conv_fwd on bf16
    input (its naive kernel) at a small size; times the C3 shape against the reference's
    fp16 WMMA kernel."""
    n, cin, cout = 3000, 256, 256
    hc, idx, ref_idx = _geometry(n, 64, 24.0, 5)
    g = torch.Generator(device=DEV).manual_seed(6)
    f = torch.randn(n, cin, device=DEV, generator=g).to(torch.bfloat16)
    w = (0.03 * torch.randn(3, 3, 3, cin, cout, device=DEV, generator=g)).to(torch.bfloat16).float()
    b = 0.1 * torch.randn(cout, device=DEV, generator=g)
    wt = w.reshape(27, cin, cout).transpose(1, 2).contiguous().to(torch.bfloat16)
    ours = fk.dense_sparse_conv3d(f, wt, b, [idx]).float()
    ref = REF.dense_conv_fwd(f, w, b, ref_idx).float()
    assert float((ours - ref).norm() / ref.norm()) < 1e-2
    # the C3 shape: ours (bf16 tcgen05) against the reference's fp16 WMMA path
    n, cin, cout = 65536, 1536, 1536
    hc, idx, ref_idx = _geometry(n, 128, 56.0, 3)
    f = torch.randn(n, cin, device=DEV, generator=g).to(torch.bfloat16)
    w = 0.02 * torch.randn(3, 3, 3, cin, cout, device=DEV, generator=g)
    b = torch.zeros(cout, device=DEV)
    wt = w.reshape(27, cin, cout).transpose(1, 2).contiguous().to(torch.bfloat16)
    f16 = f.to(torch.float16)
    t_ours = _time(lambda: fk.dense_sparse_conv3d(f, wt, b, [idx]), reps=3)
    t_ref = _time(lambda: REF.dense_conv_fwd(f16, w, b, ref_idx), reps=2)
    print(f"\ndense conv n={n} {cin}->{cout}: ours {t_ours:.2f} ms (bf16 tcgen05), reference {t_ref:.2f} ms (fp16 WMMA)")
