"""Pin the oracle's geometry on the reference's three real voxel sets.

The reference ships three public-test samples (``fetched_info/sample_test_data/
public_test/*/cache/vox_idxi.npz``, N = 4632..6082 in 64^3).  They are read in
place from a reference checkout and never copied; on a machine without the
checkout (a GPU machine, for instance) these tests skip.  The reference side is its own CPU
code: the lexicographic key sort of ``lib/fast_flow.py:675-679``,
``base_models/order.py:encode_hilbert``, ``build_order_caches_fast`` and
``build_conv_indices_fast`` (CPU fallbacks of ``lib/fast_kernels.py``).
"""
import os
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import geometry as geo

from oracle import reference_root

REF = reference_root()
SAMPLES = sorted((REF / "fetched_info" / "sample_test_data" / "public_test").glob("*/cache/vox_idxi.npz")) if REF else []

pytestmark = pytest.mark.skipif(not SAMPLES, reason="VDIT_REFERENCE_DIR does not name a reference checkout")


@pytest.fixture(scope="module")
def ref_modules():
    from tests.golden.make_golden import load_reference
    fk = load_reference(REF)
    import base_models.order as order
    return fk, order


@pytest.mark.parametrize("idx", range(3))
def test_geometry_matches_reference_on_real_voxels(ref_modules, idx):
    if idx >= len(SAMPLES):
        pytest.skip("sample missing")
    fk, order = ref_modules
    vox = np.load(SAMPLES[idx])["vox_idxi"].astype(np.int32)
    n = len(vox)

    # reference: key sort, four Hilbert codes, order caches, conv indices
    v = torch.from_numpy(vox)
    c = v.long()
    perm_ref = torch.argsort((c[:, 0] << 20) | (c[:, 1] << 10) | c[:, 2])
    hc_ref = torch.cat([torch.zeros(n, 1, dtype=torch.int32), v[perm_ref]], 1).contiguous()
    codes_ref = []
    for mode, conv in (("h", "xyz"), ("ht1", "yxz"), ("h1", "xyz"), ("ht", "yxz")):
        xyz = hc_ref.clone()
        if mode.endswith("1"):
            xyz[:, 1:] += 1
        codes_ref.append(order.encode_hilbert(xyz, conv))
    caches = fk.build_order_caches_fast(hc_ref, [n], ["h", "ht1", "h1", "ht"], {"patch_size": 4096}, {},
                                        torch.arange(n), use_triton=False)
    idx_ref = fk.build_conv_indices_fast(hc_ref, already_sorted=True)[0].numpy()

    # oracle
    perm, _, hc = geo.lex_perm(vox)
    np.testing.assert_array_equal(perm, perm_ref.numpy())
    np.testing.assert_array_equal(hc, hc_ref.numpy())
    codes = geo.encode_orders4(hc)
    np.testing.assert_array_equal(codes, torch.stack(codes_ref).numpy())
    for k, (fwd, bwd) in enumerate(geo.order_caches(codes)):
        np.testing.assert_array_equal(fwd, caches[k][0].numpy())
        np.testing.assert_array_equal(bwd, caches[k][1].numpy())
    np.testing.assert_array_equal(geo.window_cu_seqlens(n, 4096), caches[0][2].numpy())
    np.testing.assert_array_equal(geo.conv_indices(hc), idx_ref[:n])
