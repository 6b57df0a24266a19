"""The seeded synthetic workloads on CPU: exact voxel counts, unique in-grid coordinates,
and seeds that reproduce (the GPU tests, the parity cases and bench.py draw from these)."""
import numpy as np
import pytest

from vdit.workloads import C4, C5, ellipsoid_union, shell_voxels, uniform_voxels


def _check(vox: np.ndarray, n: int, grid: int):
    assert vox.shape == (n, 3) and vox.dtype == np.int32
    assert vox.min() >= 0 and vox.max() < grid
    assert len(np.unique(vox, axis=0)) == n


@pytest.mark.parametrize("seed", [0, 3, 500])
def test_ellipsoid_union_c5(seed):
    _check(ellipsoid_union(32768, 128, seed), 32768, 128)
    assert np.array_equal(ellipsoid_union(4096, 128, seed), ellipsoid_union(4096, 128, seed))


def test_shell_and_uniform():
    _check(shell_voxels(16384, 64, 36.0, 0), 16384, 64)
    _check(uniform_voxels(65536, 128, 1), 65536, 128)


def test_workload_inputs():
    w5, w4 = C5(), C4()
    assert w5.arch.res == 128 and w4.arch.res == 64 and w5.samples == 16
    a, b = w5.inputs(501, "cpu"), w5.inputs(502, "cpu")
    assert a["vox"].shape == (32768, 3) and a["context"].shape == (4101, 1536)
    assert a["noise"].shape == (32768, 16)
    assert not np.array_equal(a["vox"].numpy(), b["vox"].numpy())     # samples differ
